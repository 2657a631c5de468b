// Direct k-sum (gaussian.py:906-1081, 1180-1337) with explicit derivatives.
//   E = (1/2V) sum_{k != 0, |k| <= k_max} K(k^2) |S(k)|^2,  S(k) = sum_i q_i e^{i k.r_i}
// over the half space of integer modes n (each standing for the pair +-n);
// k = 2 pi cell^-1 n.  Forces, dE/dq, dE/d(amp, bw2) and the virial are
// explicit sums, where the reference differentiates with autograd.
//   k_direct_sfac   thread per mode: S(k) per channel, K(k), energy partials
//   k_direct_extra  parameter-gradient / virial partials (optional)
//   k_direct_atoms  thread per atom: forces and potential
#include <algorithm>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include <cuda.h>

#include "frames.cuh"
#include "plan.hpp"

namespace sogb {
namespace {

constexpr int kMaxCh = 8;
constexpr int kDirThreads = 256;

struct DirArgs {
  const FrameGeom *geom;
  const int *nk;      // [nf][3]
  int64_t kmax_modes; // stride of per-frame mode arrays
  int nch, M;
  double *kvec;       // [nf][K][4]: kx, ky, kz, K
  double *sfac;       // [nf][C][K][2]
  double *part;       // [C][nf][nblk][2]
  double *partx;      // [C][nf][nblk][4M+13]
  int nx_acc;
};

__device__ __forceinline__ bool decode_mode(int64_t t, const int *nk, int &n0, int &n1, int &n2) {
  const int w2 = 2 * nk[2] + 1, w1 = 2 * nk[1] + 1;
  n2 = (int)(t % w2) - nk[2];
  t /= w2;
  n1 = (int)(t % w1) - nk[1];
  n0 = (int)(t / w1);
  if (n0 > nk[0]) return false;
  // half space: n0 > 0 | n0 == 0 & n1 > 0 | n0 == n1 == 0 & n2 > 0
  return n0 > 0 || (n0 == 0 && (n1 > 0 || (n1 == 0 && n2 > 0)));
}

template <typename T>
__global__ void __launch_bounds__(kDirThreads) k_direct_sfac(DirArgs a, const T *__restrict__ pos,
                                                            const T *__restrict__ q,
                                                            const T *__restrict__ amp,
                                                            const T *__restrict__ bw2) {
  __shared__ double s_r[kDirThreads][3];
  __shared__ double s_q[kDirThreads][kMaxCh];
  __shared__ double s_amp[kMaxGauss], s_bw2[kMaxGauss];
  __shared__ double red[2 * kMaxCh + 1][kDirThreads / 32];
  for (int m = threadIdx.x; m < a.M; m += blockDim.x) {
    s_amp[m] = (double)amp[m];
    s_bw2[m] = (double)bw2[m];
  }
  const int f = blockIdx.y;
  const FrameGeom &g = a.geom[f];
  const int *nk = a.nk + 3 * f;
  const int64_t nbox = (int64_t)(nk[0] + 1) * (2 * nk[1] + 1) * (2 * nk[2] + 1);
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int n0 = 0, n1 = 0, n2 = 0;
  bool live = t < nbox && decode_mode(t, nk, n0, n1, n2);
  double k[3] = {0.0, 0.0, 0.0}, ksq = 0.0;
  if (live) {
    for (int c = 0; c < 3; ++c) k[c] = g.kmat[c * 3 + 0] * n0 + g.kmat[c * 3 + 1] * n1 + g.kmat[c * 3 + 2] * n2;
    ksq = k[0] * k[0] + k[1] * k[1] + k[2] * k[2];
    live = ksq <= g.k_sq_max;
  }
  __syncthreads();
  double K = 0.0;
  if (live)
    for (int m = 0; m < a.M; ++m) K += s_amp[m] * exp(-0.5 * s_bw2[m] * ksq);
  double sr[kMaxCh], si[kMaxCh];
#pragma unroll
  for (int c = 0; c < kMaxCh; ++c) { sr[c] = 0.0; si[c] = 0.0; }
  for (int base = 0; base < g.natoms; base += kDirThreads) {
    const int i = base + threadIdx.x;
    __syncthreads();
    if (i < g.natoms) {
      const int64_t atom = g.atom_begin + i;
      for (int c = 0; c < 3; ++c) s_r[threadIdx.x][c] = (double)pos[atom * 3 + c];
      for (int c = 0; c < a.nch; ++c) s_q[threadIdx.x][c] = (double)q[atom * a.nch + c];
    }
    __syncthreads();
    const int cnt = min(kDirThreads, g.natoms - base);
    if (live) {
      for (int j = 0; j < cnt; ++j) {
        const double kr = k[0] * s_r[j][0] + k[1] * s_r[j][1] + k[2] * s_r[j][2];
        double sn, cs;
        sincos(kr, &sn, &cs);
#pragma unroll
        for (int c = 0; c < kMaxCh; ++c)
          if (c < a.nch) { sr[c] += s_q[j][c] * cs; si[c] += s_q[j][c] * sn; }
      }
    }
  }
  if (t < nbox) {
    double *kv = a.kvec + ((int64_t)f * a.kmax_modes + t) * 4;
    kv[0] = k[0]; kv[1] = k[1]; kv[2] = k[2]; kv[3] = live ? K : 0.0;
    for (int c = 0; c < a.nch; ++c) {
      double *s = a.sfac + (((int64_t)f * a.nch + c) * a.kmax_modes + t) * 2;
      s[0] = live ? sr[c] : 0.0;
      s[1] = live ? si[c] : 0.0;
    }
  }
  // energy partials per channel (2 K |S|^2) and the self sum (2 K)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int c = 0; c < a.nch; ++c) {
    const double v = warp_sum(live ? 2.0 * K * (sr[c] * sr[c] + si[c] * si[c]) : 0.0);
    if (lane == 0) red[c][warp] = v;
  }
  const double dsum = warp_sum(live ? 2.0 * K : 0.0);
  if (lane == 0) red[kMaxCh * 2][warp] = dsum;
  __syncthreads();
  if (threadIdx.x < a.nch) {
    const int c = threadIdx.x;
    double e = 0.0, d = 0.0;
    for (int w = 0; w < kDirThreads / 32; ++w) { e += red[c][w]; d += red[kMaxCh * 2][w]; }
    double *p = a.part + (((int64_t)c * gridDim.y + f) * gridDim.x + blockIdx.x) * 2;
    p[0] = e;
    p[1] = d;
  }
}

// dE/d(amp, bw2) and virial partial sums; same layout as the mesh extras.
template <typename T>
__global__ void __launch_bounds__(kDirThreads) k_direct_extra(DirArgs a, const T *__restrict__ amp,
                                                             const T *__restrict__ bw2, int want_grad,
                                                             int want_vir) {
  __shared__ double s_amp[kMaxGauss], s_bw2[kMaxGauss];
  __shared__ double red[kDirThreads / 32][4 * kMaxGauss + 13];
  for (int m = threadIdx.x; m < a.M; m += blockDim.x) {
    s_amp[m] = (double)amp[m];
    s_bw2[m] = (double)bw2[m];
  }
  __syncthreads();
  const int f = blockIdx.y, c = blockIdx.z;
  const int *nk = a.nk + 3 * f;
  const int64_t nbox = (int64_t)(nk[0] + 1) * (2 * nk[1] + 1) * (2 * nk[2] + 1);
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int M = a.M;
  double k[3] = {0, 0, 0}, K = 0.0, s2 = 0.0;
  if (t < nbox) {
    const double *kv = a.kvec + ((int64_t)f * a.kmax_modes + t) * 4;
    k[0] = kv[0]; k[1] = kv[1]; k[2] = kv[2]; K = kv[3];
    const double *s = a.sfac + (((int64_t)f * a.nch + c) * a.kmax_modes + t) * 2;
    s2 = s[0] * s[0] + s[1] * s[1];
  }
  const bool live = K != 0.0;
  const double ksq = k[0] * k[0] + k[1] * k[1] + k[2] * k[2];
  if (want_grad) {
    for (int m = 0; m < M; ++m) {
      const double e = live ? exp(-0.5 * s_bw2[m] * ksq) : 0.0;
      const double hk = -0.5 * ksq * s_amp[m];
      const double v0 = warp_sum(2.0 * e * s2), v1 = warp_sum(2.0 * e);
      const double v2 = warp_sum(2.0 * hk * e * s2), v3 = warp_sum(2.0 * hk * e);
      if (lane == 0) {
        red[warp][m] = v0; red[warp][M + m] = v1; red[warp][2 * M + m] = v2; red[warp][3 * M + m] = v3;
      }
    }
  }
  if (want_vir) {
    double Kv = 0.0;
    if (live)
      for (int m = 0; m < M; ++m) Kv += s_amp[m] * s_bw2[m] * exp(-0.5 * s_bw2[m] * ksq);
    const double kk[6] = {k[0] * k[0], k[1] * k[1], k[2] * k[2], k[0] * k[1], k[0] * k[2], k[1] * k[2]};
    double v = warp_sum(2.0 * s2 * K);
    if (lane == 0) red[warp][4 * M] = v;
    for (int q = 0; q < 6; ++q) {
      v = warp_sum(live ? 2.0 * s2 * Kv * kk[q] : 0.0);
      if (lane == 0) red[warp][4 * M + 1 + q] = v;
      v = warp_sum(live ? 2.0 * Kv * kk[q] : 0.0);
      if (lane == 0) red[warp][4 * M + 7 + q] = v;
    }
  }
  __syncthreads();
  const int nacc = 4 * M + 13;
  double *p = a.partx + (((int64_t)c * gridDim.y + f) * gridDim.x + blockIdx.x) * a.nx_acc;
  for (int i = threadIdx.x; i < nacc; i += blockDim.x) {
    const bool used = (i < 4 * M) ? want_grad : want_vir;
    double s = 0.0;
    if (used)
      for (int w = 0; w < kDirThreads / 32; ++w) s += red[w][i];
    p[i] = s;
  }
}

// CH threads per block, one atom each, staging CH modes at a time: 128, or
// one warp for frames of at most 32 atoms (many tiny frames), so that a
// block's threads are mostly busy.
template <typename T, int CH = 128>
__global__ void __launch_bounds__(CH) k_direct_atoms(DirArgs a, const T *__restrict__ pos,
                                                    const T *__restrict__ q, double norm,
                                                    T *__restrict__ forces, T *__restrict__ pot) {
  __shared__ double s_k[CH][4];
  __shared__ double s_s[CH][kMaxCh][2];
  const int f = blockIdx.y;
  const FrameGeom &g = a.geom[f];
  const int *nk = a.nk + 3 * f;
  const int64_t nbox = (int64_t)(nk[0] + 1) * (2 * nk[1] + 1) * (2 * nk[2] + 1);
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const bool own = i < g.natoms;
  const int64_t atom = g.atom_begin + (own ? i : 0);
  double r[3] = {0, 0, 0}, qi[kMaxCh];
  if (own)
    for (int c = 0; c < 3; ++c) r[c] = (double)pos[atom * 3 + c];
#pragma unroll
  for (int c = 0; c < kMaxCh; ++c) qi[c] = (own && c < a.nch) ? (double)q[atom * a.nch + c] : 0.0;
  double fx = 0, fy = 0, fz = 0, pc[kMaxCh];
#pragma unroll
  for (int c = 0; c < kMaxCh; ++c) pc[c] = 0.0;
  for (int64_t base = 0; base < nbox; base += CH) {
    __syncthreads();
    const int64_t t = base + threadIdx.x;
    if (t < nbox) {
      const double *kv = a.kvec + ((int64_t)f * a.kmax_modes + t) * 4;
      for (int c = 0; c < 4; ++c) s_k[threadIdx.x][c] = kv[c];
      for (int c = 0; c < a.nch; ++c) {
        const double *s = a.sfac + (((int64_t)f * a.nch + c) * a.kmax_modes + t) * 2;
        s_s[threadIdx.x][c][0] = s[0];
        s_s[threadIdx.x][c][1] = s[1];
      }
    } else {
      s_k[threadIdx.x][3] = 0.0;
    }
    __syncthreads();
    const int cnt = (int)min((int64_t)CH, nbox - base);
    if (own) {
      for (int j = 0; j < cnt; ++j) {
        const double K = s_k[j][3];
        if (K == 0.0) continue;
        const double kr = s_k[j][0] * r[0] + s_k[j][1] * r[1] + s_k[j][2] * r[2];
        double sn, cs;
        sincos(kr, &sn, &cs);
        double tsum = 0.0;
#pragma unroll
        for (int c = 0; c < kMaxCh; ++c) {
          if (c < a.nch) {
            const double sr = s_s[j][c][0], si = s_s[j][c][1];
            tsum += qi[c] * (si * cs - sr * sn);
            pc[c] += 2.0 * K * (sr * cs + si * sn);
          }
        }
        const double tt = 2.0 * K * tsum;
        fx += tt * s_k[j][0];
        fy += tt * s_k[j][1];
        fz += tt * s_k[j][2];
      }
    }
  }
  if (!own) return;
  if (forces) {
    const double sc = -norm / g.vol;
    forces[atom * 3 + 0] = (T)(sc * fx);
    forces[atom * 3 + 1] = (T)(sc * fy);
    forces[atom * 3 + 2] = (T)(sc * fz);
  }
  if (pot)
    for (int c = 0; c < a.nch; ++c) pot[atom * a.nch + c] = (T)(pc[c] / g.vol);
}

inline unsigned nblk(int64_t n, int b) { return (unsigned)((n + b - 1) / b); }

inline void after(Tracer *tr, cudaStream_t st, const char *name) {
  count_launch();
  if (tr) tr->mark(st, name);
}

template <typename T>
int direct_impl(sog_direct *d, const sog_direct_args *a, cudaStream_t st) {
  const int nf = a->nframes, nch = a->nchannels, M = a->n_gauss;
  std::vector<FrameHost> fh(nf);
  int64_t kmax = 1, maxat = 0, slots = 0;
  for (int f = 0; f < nf; ++f) {
    for (int c = 0; c < 3; ++c)
      if (a->nk[3 * f + c] < 0 || a->nk[3 * f + c] > 4096) return fail(SOG_ERR_INVALID, "nk out of range");
    const int64_t nbox = (int64_t)(a->nk[3 * f] + 1) * (2 * a->nk[3 * f + 1] + 1) * (2 * a->nk[3 * f + 2] + 1);
    kmax = std::max(kmax, nbox);
    maxat = std::max<int64_t>(maxat, a->atom_count[f]);
    fh[f].atom_begin = a->atom_begin[f];
    fh[f].natoms = a->atom_count[f];
    fh[f].slot_base = slots;
    fh[f].k_sq_max = a->k_sq_max[f];
    slots += a->atom_count[f];
  }
  if (kmax > ((int64_t)1 << 31)) return fail(SOG_ERR_INVALID, "mode box too large");
  const unsigned kb = nblk(kmax, kDirThreads);
  const int nx_acc = 4 * M + 13;
  const bool want_grad = a->grad_amp || a->grad_bw2;
  const bool want_vir = a->virial != nullptr;
  int rc;
  if ((rc = d->up.reserve(sizeof(FrameHost) * nf + sizeof(int) * 3 * nf)) != SOG_OK) return rc;
  if ((rc = d->up.wait()) != SOG_OK) return rc;
  std::memcpy(d->up.p, fh.data(), sizeof(FrameHost) * nf);
  std::memcpy((char *)d->up.p + sizeof(FrameHost) * nf, a->nk, sizeof(int) * 3 * nf);
  if (d->frames_host_dev.reserve(sizeof(FrameHost) * nf + sizeof(int) * 3 * nf) ||
      d->geom.reserve(sizeof(FrameGeom) * nf) || d->status.reserve(16) ||
      d->modes.reserve(sizeof(double) * 4 * kmax * nf) ||
      d->sfac.reserve(sizeof(double) * 2 * kmax * nf * nch) ||
      d->part.reserve(sizeof(double) * ((int64_t)2 + ((want_grad || want_vir) ? nx_acc : 0)) * kb * nf * nch +
                      sizeof(double) * ((int64_t)nf * nch * (2 + nx_acc) + (int64_t)nf * 4)) ||
      d->qsum.reserve(sizeof(double) * 2 * nf * nch))
    return fail(SOG_ERR_NOMEM, "device allocation failed (direct)");
  SOG_CUDA_TRY(cudaMemcpyAsync(d->frames_host_dev.p, d->up.p, sizeof(FrameHost) * nf + sizeof(int) * 3 * nf,
                               cudaMemcpyHostToDevice, st));
  SOG_CUDA_TRY(cudaEventRecord(d->up.done, st));
  d->up.pending = true;
  FrameGeom *geom = d->geom.as<FrameGeom>();
  const FrameHost *fhd = d->frames_host_dev.as<FrameHost>();
  const int *nkd = reinterpret_cast<const int *>(fhd + nf);
  Tracer *tr = &d->tr;
  tr->begin(st);
  k_frame_setup<T><<<nblk(nf, 128), 128, 0, st>>>((const T *)a->cells, fhd, geom, nf, SOG_KCONV_PHYSICAL,
                                                  1, 1, 1, d->status.as<unsigned>());
  after(tr, st, "frame_setup");
  const int qs = (int)std::max<int64_t>(1, std::min<int64_t>(256, (maxat + 16383) / 16384));
  if (d->qpart.reserve(sizeof(double) * 2 * (int64_t)nf * nch * qs) ||
      d->redtmp.reserve(sizeof(double) * std::max(reduce_tmp_elems(nf, nch, kb, 2),
                                                   reduce_tmp_elems(nf, nch, kb, nx_acc))))
    return fail(SOG_ERR_NOMEM, "device allocation failed (direct)");
  k_qsums<T><<<dim3(nf, nch, qs), 256, 0, st>>>((const T *)a->charges, nch, geom, d->qpart.as<double>(),
                                                (const T *)a->positions, d->status.as<unsigned>());
  k_reduce_parts<<<dim3(nf, nch, 1), 256, 0, st>>>(d->qpart.as<double>(), nf, nch, qs, 2, 2,
                                                  d->qsum.as<double>());
  after(tr, st, "qsums");
  count_launch();
  DirArgs da;
  da.geom = geom;
  da.nk = nkd;
  da.kmax_modes = kmax;
  da.nch = nch;
  da.M = M;
  da.kvec = d->modes.as<double>();
  da.sfac = d->sfac.as<double>();
  da.part = d->part.as<double>();
  da.partx = da.part + (int64_t)2 * kb * nf * nch;
  da.nx_acc = nx_acc;
  double *redE = da.partx + ((want_grad || want_vir) ? (int64_t)nx_acc * kb * nf * nch : 0);
  double *redX = redE + (int64_t)nf * nch * 2;
  double *fscal = redX + (int64_t)nf * nch * nx_acc;
  k_direct_sfac<T><<<dim3(kb, nf), kDirThreads, 0, st>>>(da, (const T *)a->positions, (const T *)a->charges,
                                                         (const T *)a->amp, (const T *)a->bw2);
  after(tr, st, "direct_sfac");
  if (want_grad || want_vir)
    k_direct_extra<T><<<dim3(kb, nf, nch), kDirThreads, 0, st>>>(da, (const T *)a->amp, (const T *)a->bw2,
                                                                 want_grad, want_vir);
  if (want_grad || want_vir) after(tr, st, "direct_extra");
  if ((a->forces || a->potential) && maxat > 0) {
    if (maxat <= 32)
      k_direct_atoms<T, 32><<<dim3(1, nf), 32, 0, st>>>(da, (const T *)a->positions, (const T *)a->charges,
                                                        a->norm_factor, (T *)a->forces, (T *)a->potential);
    else
      k_direct_atoms<T><<<dim3(nblk(maxat, 128), nf), 128, 0, st>>>(da, (const T *)a->positions,
                                                                    (const T *)a->charges, a->norm_factor,
                                                                    (T *)a->forces, (T *)a->potential);
  }
  if ((a->forces || a->potential) && maxat > 0) after(tr, st, "direct_atoms");
  reduce_parts(da.part, nf, nch, kb, 2, 2, redE, d->redtmp.as<double>(), st);
  after(tr, st, "reduce");
  if (reduce_split(kb) > 1) count_launch();
  if (want_grad || want_vir)
    reduce_parts(da.partx, nf, nch, kb, nx_acc, nx_acc, redX, d->redtmp.as<double>(), st);
  if (want_grad || want_vir) {
    after(tr, st, "reduce_extra");
    if (reduce_split(kb) > 1) count_launch();
  }
  FinalArgs fa;
  std::memset(&fa, 0, sizeof(fa));
  fa.geom = geom;
  fa.redE = redE;
  fa.redX = redX;
  fa.qsum = d->qsum.as<double>();
  fa.amp = a->amp;
  fa.bw2 = a->bw2;
  fa.M = M; fa.nch = nch; fa.nx = 1; fa.ny = 1; fa.nz = 1;
  fa.norm = a->norm_factor;
  fa.self_coeff = a->self_coeff;
  fa.lambda = a->charge_neutral_lambda;
  fa.remove_self = a->remove_self;
  fa.k0 = a->k0_correction;
  fa.want_grad = want_grad;
  fa.want_vir = want_vir;
  fa.direct = 1;
  fa.energy = a->energy;
  fa.grad_amp = a->grad_amp;
  fa.grad_bw2 = a->grad_bw2;
  fa.virial = a->virial;
  fa.fscal = fscal;
  k_finalize_frames<T><<<nblk(nf, 64), 64, 0, st>>>(fa, nf);
  after(tr, st, "finalize_frames");
  if (a->potential && maxat > 0)
    k_finalize_atoms<T><<<dim3(nblk(maxat, 256), nf), 256, 0, st>>>(
        geom, fscal, d->qsum.as<double>(), (const T *)a->charges, (T *)a->potential, nch, a->norm_factor,
        a->self_coeff, a->charge_neutral_lambda, a->remove_self, a->k0_correction);
  if (a->potential && maxat > 0) after(tr, st, "finalize_atoms");
  SOG_CUDA_TRY(cudaGetLastError());
  return SOG_OK;
}

}  // namespace
}  // namespace sogb

using namespace sogb;

extern "C" int sog_direct_create(sog_direct **out, int dtype, int device) {
  if (!out) return fail(SOG_ERR_INVALID, "null argument");
  if (dtype != SOG_DTYPE_F64 && dtype != SOG_DTYPE_F32) return fail(SOG_ERR_INVALID, "bad dtype");
  sog_direct *d = new sog_direct();
  d->dtype = dtype;
  d->device = device;
  *out = d;
  return SOG_OK;
}

extern "C" int sog_direct_destroy(sog_direct *d) {
  if (!d) return SOG_OK;
  DeviceGuard dg(d->device);
  DevBuf *bufs[] = {&d->frames_host_dev, &d->geom, &d->modes, &d->sfac, &d->part, &d->qsum, &d->status,
                    &d->qpart, &d->redtmp, &d->hx, &d->hpart, &d->hred, &d->hdsum, &d->hscal};
  for (DevBuf *b : bufs) b->release();
  d->up.release();
  d->tr.release();
  delete d;
  return SOG_OK;
}

extern "C" int sog_direct_forward(sog_direct *d, const sog_direct_args *a, void *stream) {
  if (!d || !a) return fail(SOG_ERR_INVALID, "null argument");
  if (a->nframes <= 0) return SOG_OK;
  if (!a->atom_begin || !a->atom_count || !a->nk || !a->k_sq_max || !a->positions || !a->charges ||
      !a->cells || !a->amp || !a->bw2)
    return fail(SOG_ERR_INVALID, "missing input array");
  if (a->nchannels < 1 || a->nchannels > kMaxCh)
    return fail(SOG_ERR_UNSUPPORTED, "direct k-sum supports 1..8 charge channels");
  if (a->n_gauss < 1 || a->n_gauss > kMaxGauss) return fail(SOG_ERR_INVALID, "n_gauss must be in [1, 64]");
  DeviceGuard dg(d->device);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (d->dtype == SOG_DTYPE_F64) return direct_impl<double>(d, a, st);
  return direct_impl<float>(d, a, st);
}

// ==========================================================================
// Hessian-vector products of the direct k-sum (double backward).
//
// With E = beta sum_half K |S|^2 (beta = 1/V), S = sum_j q_j e_j, e_j =
// exp(i k.r_j), and a direction (a_j on the charges, b_j on the positions,
// c on the kernel parameters):
//   S_d = sum_j (a_j + i q_j k.b_j) e_j,   dK = sum_m c . dK/d(amp_m, bw2_m),
//   X   = K S_d + dK S,
//   (H d)_{q_j}  = 2 beta sum [Re(conj X e_j) - K (k.b_j) Im(conj S e_j)]
//   (H d)_{r_j}  = -2 beta sum k [q_j Im(conj X e_j) + a_j K Im(conj S e_j)
//                                 + q_j K (k.b_j) Re(conj S e_j)]
//   (H d)_{theta_m} = beta sum [2 dK/dtheta_m Re(conj S S_d) + d(dK)/dtheta_m |S|^2]
// per channel (positions shared).  The self, k=0 and penalty terms depend on
// the charges and parameters only; their exact second derivatives are added
// per frame and per atom from the mode sums D0..D2 of exp(-bw2_m k^2 / 2).
// ==========================================================================
namespace sogb {
namespace {

struct HvpArgs {
  const void *dq, *dr, *damp, *dbw2;  // directions (null: zero)
  void *oq, *orr, *oamp, *obw2;       // outputs
  double *hx;                          // [nf][C][K][2] X sums
  double *hpart;                       // [nf][nblk][5M] partials: 2M theta rows, D0, D1, D2
  int nh;                              // 5M
};

// thread per mode: S_d, X = K S_d + dK S, theta partials and the D sums
template <typename T>
__global__ void __launch_bounds__(kDirThreads) k_direct_hvp_modes(DirArgs a, HvpArgs h, const T *__restrict__ pos,
                                                                 const T *__restrict__ q, const T *__restrict__ amp,
                                                                 const T *__restrict__ bw2) {
  __shared__ double s_r[kDirThreads][3];
  __shared__ double s_b[kDirThreads][3];
  __shared__ double s_q[kDirThreads][kMaxCh];
  __shared__ double s_a[kDirThreads][kMaxCh];
  __shared__ double s_amp[kMaxGauss], s_bw2[kMaxGauss], s_ca[kMaxGauss], s_cb[kMaxGauss];
  __shared__ double red[kDirThreads / 32];
  const int f = blockIdx.y;
  const FrameGeom &g = a.geom[f];
  for (int m = threadIdx.x; m < a.M; m += blockDim.x) {
    s_amp[m] = (double)amp[m];
    s_bw2[m] = (double)bw2[m];
    s_ca[m] = ldir<T>(h.damp, (int64_t)f * a.M + m);
    s_cb[m] = ldir<T>(h.dbw2, (int64_t)f * a.M + m);
  }
  __syncthreads();
  const int *nk = a.nk + 3 * f;
  const int64_t nbox = (int64_t)(nk[0] + 1) * (2 * nk[1] + 1) * (2 * nk[2] + 1);
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  double k[3] = {0.0, 0.0, 0.0}, K = 0.0;
  if (t < nbox) {
    const double *kv = a.kvec + ((int64_t)f * a.kmax_modes + t) * 4;
    k[0] = kv[0]; k[1] = kv[1]; k[2] = kv[2]; K = kv[3];
  }
  const bool live = K != 0.0;
  const double ksq = k[0] * k[0] + k[1] * k[1] + k[2] * k[2];
  double dr[kMaxCh], di[kMaxCh];
#pragma unroll
  for (int c = 0; c < kMaxCh; ++c) { dr[c] = 0.0; di[c] = 0.0; }
  for (int base = 0; base < g.natoms; base += kDirThreads) {
    const int i = base + threadIdx.x;
    __syncthreads();
    if (i < g.natoms) {
      const int64_t atom = g.atom_begin + i;
      for (int c = 0; c < 3; ++c) {
        s_r[threadIdx.x][c] = (double)pos[atom * 3 + c];
        s_b[threadIdx.x][c] = ldir<T>(h.dr, atom * 3 + c);
      }
      for (int c = 0; c < a.nch; ++c) {
        s_q[threadIdx.x][c] = (double)q[atom * a.nch + c];
        s_a[threadIdx.x][c] = ldir<T>(h.dq, atom * a.nch + c);
      }
    }
    __syncthreads();
    const int cnt = min(kDirThreads, g.natoms - base);
    if (live) {
      for (int j = 0; j < cnt; ++j) {
        const double kr = k[0] * s_r[j][0] + k[1] * s_r[j][1] + k[2] * s_r[j][2];
        const double kb = k[0] * s_b[j][0] + k[1] * s_b[j][1] + k[2] * s_b[j][2];
        double sn, cs;
        sincos(kr, &sn, &cs);
#pragma unroll
        for (int c = 0; c < kMaxCh; ++c)
          if (c < a.nch) {
            const double av = s_a[j][c], qk = s_q[j][c] * kb;
            dr[c] += av * cs - qk * sn;
            di[c] += av * sn + qk * cs;
          }
      }
    }
  }
  // dK of the direction and the per-Gaussian factors
  double dK = 0.0;
  if (live)
    for (int m = 0; m < a.M; ++m)
      dK += (s_ca[m] - 0.5 * ksq * s_amp[m] * s_cb[m]) * exp(-0.5 * s_bw2[m] * ksq);
  double rsd = 0.0, s2 = 0.0;   // sum_c Re(conj S S_d), sum_c |S|^2
  if (t < nbox) {
    for (int c = 0; c < a.nch; ++c) {
      const double *sp = a.sfac + (((int64_t)f * a.nch + c) * a.kmax_modes + t) * 2;
      const double sr = sp[0], si = sp[1];
      rsd += sr * dr[c] + si * di[c];
      s2 += sr * sr + si * si;
      double *xp = h.hx + (((int64_t)f * a.nch + c) * a.kmax_modes + t) * 2;
      xp[0] = live ? K * dr[c] + dK * sr : 0.0;
      xp[1] = live ? K * di[c] + dK * si : 0.0;
    }
  }
  // partials: theta rows (amp, bw2) and the D sums, over the half space
  // (weights 2 as k_direct_sfac's energy sums; scaled on the host side)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int M = a.M;
  double *out = h.hpart + ((int64_t)f * gridDim.x + blockIdx.x) * h.nh;
  for (int m = 0; m < M; ++m) {
    const double e = live ? exp(-0.5 * s_bw2[m] * ksq) : 0.0;
    const double hk = -0.5 * ksq;
    const double v[5] = {
        2.0 * (2.0 * e * rsd + s_cb[m] * hk * e * s2),
        2.0 * (2.0 * hk * s_amp[m] * e * rsd + (s_ca[m] * hk * e + s_cb[m] * hk * hk * s_amp[m] * e) * s2),
        2.0 * e, 2.0 * hk * e, 2.0 * hk * hk * e};
#pragma unroll
    for (int r = 0; r < 5; ++r) {
      const double w = warp_sum(v[r]);
      __syncthreads();
      if (lane == 0) red[warp] = w;
      __syncthreads();
      if (threadIdx.x == 0) {
        double sacc = 0.0;
        for (int wi = 0; wi < kDirThreads / 32; ++wi) sacc += red[wi];
        out[r * M + m] = sacc;
      }
    }
  }
}

// thread per atom: the charge and position rows of H d (core term)
template <typename T, int CH = 128>
__global__ void __launch_bounds__(CH) k_direct_hvp_atoms(DirArgs a, HvpArgs h, const T *__restrict__ pos,
                                                        const T *__restrict__ q, double norm) {
  __shared__ double s_k[CH][4];
  __shared__ double s_s[CH][kMaxCh][2];
  __shared__ double s_x[CH][kMaxCh][2];
  const int f = blockIdx.y;
  const FrameGeom &g = a.geom[f];
  const int *nk = a.nk + 3 * f;
  const int64_t nbox = (int64_t)(nk[0] + 1) * (2 * nk[1] + 1) * (2 * nk[2] + 1);
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const bool own = i < g.natoms;
  const int64_t atom = g.atom_begin + (own ? i : 0);
  double r[3] = {0, 0, 0}, b[3] = {0, 0, 0}, qi[kMaxCh], ai[kMaxCh];
  if (own)
    for (int c = 0; c < 3; ++c) {
      r[c] = (double)pos[atom * 3 + c];
      b[c] = ldir<T>(h.dr, atom * 3 + c);
    }
#pragma unroll
  for (int c = 0; c < kMaxCh; ++c) {
    qi[c] = (own && c < a.nch) ? (double)q[atom * a.nch + c] : 0.0;
    ai[c] = (own && c < a.nch) ? ldir<T>(h.dq, atom * a.nch + c) : 0.0;
  }
  double px[kMaxCh], bs[kMaxCh];
#pragma unroll
  for (int c = 0; c < kMaxCh; ++c) { px[c] = 0.0; bs[c] = 0.0; }
  double fr[3] = {0, 0, 0};   // sum k (q Im X + a K Im S + q K kb Re S)
  for (int64_t base = 0; base < nbox; base += CH) {
    __syncthreads();
    const int64_t t = base + threadIdx.x;
    if (t < nbox) {
      const double *kv = a.kvec + ((int64_t)f * a.kmax_modes + t) * 4;
      for (int c = 0; c < 4; ++c) s_k[threadIdx.x][c] = kv[c];
      for (int c = 0; c < a.nch; ++c) {
        const int64_t o = (((int64_t)f * a.nch + c) * a.kmax_modes + t) * 2;
        s_s[threadIdx.x][c][0] = a.sfac[o];
        s_s[threadIdx.x][c][1] = a.sfac[o + 1];
        s_x[threadIdx.x][c][0] = h.hx[o];
        s_x[threadIdx.x][c][1] = h.hx[o + 1];
      }
    } else {
      s_k[threadIdx.x][3] = 0.0;
    }
    __syncthreads();
    const int cnt = (int)min((int64_t)CH, nbox - base);
    if (own) {
      for (int j = 0; j < cnt; ++j) {
        const double K = s_k[j][3];
        if (K == 0.0) continue;
        const double kr = s_k[j][0] * r[0] + s_k[j][1] * r[1] + s_k[j][2] * r[2];
        const double kb = s_k[j][0] * b[0] + s_k[j][1] * b[1] + s_k[j][2] * b[2];
        double sn, cs;
        sincos(kr, &sn, &cs);
        double tsum = 0.0;
#pragma unroll
        for (int c = 0; c < kMaxCh; ++c) {
          if (c < a.nch) {
            const double sr = s_s[j][c][0], si = s_s[j][c][1];
            const double xr = s_x[j][c][0], xi = s_x[j][c][1];
            const double reS = sr * cs + si * sn, imS = sr * sn - si * cs;
            const double reX = xr * cs + xi * sn, imX = xr * sn - xi * cs;
            px[c] += reX;
            bs[c] += K * kb * imS;
            tsum += qi[c] * imX + ai[c] * K * imS + qi[c] * K * kb * reS;
          }
        }
        fr[0] += tsum * s_k[j][0];
        fr[1] += tsum * s_k[j][1];
        fr[2] += tsum * s_k[j][2];
      }
    }
  }
  if (!own) return;
  const double sc = 2.0 * norm / g.vol;
  T *oq = static_cast<T *>(h.oq), *orr = static_cast<T *>(h.orr);
  for (int c = 0; c < a.nch; ++c) oq[atom * a.nch + c] = (T)(sc * (px[c] - bs[c]));
  for (int c = 0; c < 3; ++c) orr[atom * 3 + c] = (T)(-sc * fr[c]);
}

template <typename T>
int direct_hvp_impl(sog_direct *d, const sog_direct_args *a, const sog_hvp_args *hv, cudaStream_t st) {
  const int nf = a->nframes, nch = a->nchannels, M = a->n_gauss;
  std::vector<FrameHost> fh(nf);
  int64_t kmax = 1, maxat = 0, slots = 0;
  for (int f = 0; f < nf; ++f) {
    for (int c = 0; c < 3; ++c)
      if (a->nk[3 * f + c] < 0 || a->nk[3 * f + c] > 4096) return fail(SOG_ERR_INVALID, "nk out of range");
    const int64_t nbox = (int64_t)(a->nk[3 * f] + 1) * (2 * a->nk[3 * f + 1] + 1) * (2 * a->nk[3 * f + 2] + 1);
    kmax = std::max(kmax, nbox);
    maxat = std::max<int64_t>(maxat, a->atom_count[f]);
    fh[f].atom_begin = a->atom_begin[f];
    fh[f].natoms = a->atom_count[f];
    fh[f].slot_base = slots;
    fh[f].k_sq_max = a->k_sq_max[f];
    slots += a->atom_count[f];
  }
  if (kmax > ((int64_t)1 << 31)) return fail(SOG_ERR_INVALID, "mode box too large");
  const unsigned kb = nblk(kmax, kDirThreads);
  const int nh = 5 * M;
  int rc;
  if ((rc = d->up.reserve(sizeof(FrameHost) * nf + sizeof(int) * 3 * nf)) != SOG_OK) return rc;
  if ((rc = d->up.wait()) != SOG_OK) return rc;
  std::memcpy(d->up.p, fh.data(), sizeof(FrameHost) * nf);
  std::memcpy((char *)d->up.p + sizeof(FrameHost) * nf, a->nk, sizeof(int) * 3 * nf);
  const int qs = (int)std::max<int64_t>(1, std::min<int64_t>(256, (maxat + 16383) / 16384));
  if (d->frames_host_dev.reserve(sizeof(FrameHost) * nf + sizeof(int) * 3 * nf) ||
      d->geom.reserve(sizeof(FrameGeom) * nf) || d->status.reserve(16) ||
      d->modes.reserve(sizeof(double) * 4 * kmax * nf) || d->sfac.reserve(sizeof(double) * 2 * kmax * nf * nch) ||
      d->part.reserve(sizeof(double) * 2 * kb * nf * nch) || d->qsum.reserve(sizeof(double) * 2 * nf * nch) ||
      d->qpart.reserve(sizeof(double) * 2 * (int64_t)nf * nch * qs) ||
      d->hx.reserve(sizeof(double) * 2 * kmax * nf * nch) || d->hpart.reserve(sizeof(double) * nh * kb * nf) ||
      d->hred.reserve(sizeof(double) * nh * nf) || d->hdsum.reserve(sizeof(double) * 2 * nf * nch) ||
      d->hscal.reserve(sizeof(double) * 8 * nf) ||
      d->redtmp.reserve(sizeof(double) * std::max<int64_t>(reduce_tmp_elems(nf, 1, kb, nh), 1)))
    return fail(SOG_ERR_NOMEM, "device allocation failed (direct HVP)");
  SOG_CUDA_TRY(cudaMemcpyAsync(d->frames_host_dev.p, d->up.p, sizeof(FrameHost) * nf + sizeof(int) * 3 * nf,
                               cudaMemcpyHostToDevice, st));
  SOG_CUDA_TRY(cudaEventRecord(d->up.done, st));
  d->up.pending = true;
  FrameGeom *geom = d->geom.as<FrameGeom>();
  const FrameHost *fhd = d->frames_host_dev.as<FrameHost>();
  const int *nkd = reinterpret_cast<const int *>(fhd + nf);
  Tracer *tr = &d->tr;
  tr->begin(st);
  k_frame_setup<T><<<nblk(nf, 128), 128, 0, st>>>((const T *)a->cells, fhd, geom, nf, SOG_KCONV_PHYSICAL, 1, 1, 1,
                                                  d->status.as<unsigned>());
  after(tr, st, "frame_setup");
  k_qsums<T><<<dim3(nf, nch, qs), 256, 0, st>>>((const T *)a->charges, nch, geom, d->qpart.as<double>());
  k_reduce_parts<<<dim3(nf, nch, 1), 256, 0, st>>>(d->qpart.as<double>(), nf, nch, qs, 2, 2, d->qsum.as<double>());
  after(tr, st, "qsums");
  count_launch();
  DirArgs da;
  da.geom = geom;
  da.nk = nkd;
  da.kmax_modes = kmax;
  da.nch = nch;
  da.M = M;
  da.kvec = d->modes.as<double>();
  da.sfac = d->sfac.as<double>();
  da.part = d->part.as<double>();
  da.partx = nullptr;
  da.nx_acc = 0;
  k_direct_sfac<T><<<dim3(kb, nf), kDirThreads, 0, st>>>(da, (const T *)a->positions, (const T *)a->charges,
                                                         (const T *)a->amp, (const T *)a->bw2);
  after(tr, st, "direct_sfac");
  HvpArgs h;
  h.dq = hv->dir_q;
  h.dr = hv->dir_r;
  h.damp = hv->dir_amp;
  h.dbw2 = hv->dir_bw2;
  h.oq = hv->out_q;
  h.orr = hv->out_r;
  h.oamp = hv->out_amp;
  h.obw2 = hv->out_bw2;
  h.hx = d->hx.as<double>();
  h.hpart = d->hpart.as<double>();
  h.nh = nh;
  k_direct_hvp_modes<T><<<dim3(kb, nf), kDirThreads, 0, st>>>(da, h, (const T *)a->positions,
                                                              (const T *)a->charges, (const T *)a->amp,
                                                              (const T *)a->bw2);
  after(tr, st, "hvp_modes");
  if (maxat > 0) {
    if (maxat <= 32)
      k_direct_hvp_atoms<T, 32><<<dim3(1, nf), 32, 0, st>>>(da, h, (const T *)a->positions, (const T *)a->charges,
                                                            a->norm_factor);
    else
      k_direct_hvp_atoms<T><<<dim3(nblk(maxat, 128), nf), 128, 0, st>>>(da, h, (const T *)a->positions,
                                                                        (const T *)a->charges, a->norm_factor);
    after(tr, st, "hvp_atoms");
  }
  reduce_parts(h.hpart, nf, 1, kb, nh, nh, d->hred.as<double>(), d->redtmp.as<double>(), st);
  after(tr, st, "reduce");
  if (reduce_split(kb) > 1) count_launch();
  k_hvp_dsums<T><<<dim3(nf, nch), 256, 0, st>>>((const T *)a->charges, hv->dir_q, nch, geom, d->hdsum.as<double>());
  after(tr, st, "hvp_dsums");
  HvpFinal hf;
  hf.geom = geom;
  hf.hred = d->hred.as<double>();
  hf.qsum = d->qsum.as<double>();
  hf.dsum = d->hdsum.as<double>();
  hf.amp = a->amp;
  hf.bw2 = a->bw2;
  hf.damp = hv->dir_amp;
  hf.dbw2 = hv->dir_bw2;
  hf.oamp = hv->out_amp;
  hf.obw2 = hv->out_bw2;
  hf.scal = d->hscal.as<double>();
  hf.M = M;
  hf.nch = nch;
  hf.norm = a->norm_factor;
  hf.self_coeff = a->self_coeff;
  hf.lambda = a->charge_neutral_lambda;
  hf.remove_self = a->remove_self;
  hf.k0 = a->k0_correction;
  k_hvp_finalize_frames<T><<<nblk(nf, 64), 64, 0, st>>>(hf, nf);
  after(tr, st, "hvp_finalize_frames");
  if (maxat > 0) {
    k_hvp_finalize_atoms<T><<<dim3(nblk(maxat, 256), nf), 256, 0, st>>>(
        geom, d->hscal.as<double>(), d->hdsum.as<double>(), (const T *)a->charges, hv->dir_q, (T *)hv->out_q, nch,
        a->norm_factor, a->charge_neutral_lambda);
    after(tr, st, "hvp_finalize_atoms");
  }
  SOG_CUDA_TRY(cudaGetLastError());
  return SOG_OK;
}

}  // namespace
}  // namespace sogb

extern "C" int sog_direct_hvp(sog_direct *d, const sog_direct_args *a, const sog_hvp_args *h, void *stream) {
  if (!d || !a || !h) return fail(SOG_ERR_INVALID, "null argument");
  if (a->nframes <= 0) return SOG_OK;
  if (!a->atom_begin || !a->atom_count || !a->nk || !a->k_sq_max || !a->positions || !a->charges ||
      !a->cells || !a->amp || !a->bw2)
    return fail(SOG_ERR_INVALID, "missing input array");
  if (!h->out_q || !h->out_r || !h->out_amp || !h->out_bw2) return fail(SOG_ERR_INVALID, "missing HVP output array");
  if (a->nchannels < 1 || a->nchannels > kMaxCh)
    return fail(SOG_ERR_UNSUPPORTED, "direct k-sum supports 1..8 charge channels");
  if (a->n_gauss < 1 || a->n_gauss > kMaxGauss) return fail(SOG_ERR_INVALID, "n_gauss must be in [1, 64]");
  DeviceGuard dg(d->device);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (d->dtype == SOG_DTYPE_F64) return direct_hvp_impl<double>(d, a, h, st);
  return direct_hvp_impl<float>(d, a, h, st);
}

// ==========================================================================
// No-allocation variant of the direct k-sum.
//
// Some callers cannot allocate device or pinned memory inside their force
// call: an MD engine that hands out device memory only from its own arena
// and forbids cudaMalloc after setup (cudaMalloc and cudaHostAlloc can block
// on work already queued on the device and can fail under memory pressure in
// the middle of a run), or an integrator that must not create per-context
// state.  sog_direct_forward_noalloc runs the same kernels as
// sog_direct_forward with all scratch in one fixed file-scope device array
// and the per-frame metadata passed by value as a kernel parameter, so a
// call makes no allocation of any kind.
//
// Limits: SOG_NOALLOC_SCRATCH_BYTES of scratch per device and at most
// SOG_NOALLOC_MAX_FRAMES frames per call; a call that needs more is rejected
// with SOG_ERR_INVALID before anything is launched.  Nothing in the scratch
// has to start at zero: every word a call reads was written earlier in the
// same call (the status word is cleared by the call's first kernel).  The
// scratch is shared by every call on a device, so two calls in flight at
// once on one device (different streams or host threads) race; callers
// serialise them (one stream, or an event between them).
// ==========================================================================
namespace sogb {
namespace {

constexpr size_t kNoAllocBytes = SOG_NOALLOC_SCRATCH_BYTES;
constexpr int kNoAllocFrames = SOG_NOALLOC_MAX_FRAMES;

static __device__ __align__(256) unsigned char g_direct_scratch[kNoAllocBytes];

struct NoAllocFrames {
  FrameHost fh[kNoAllocFrames];
  int nk[kNoAllocFrames][3];
  int nf;
};
static_assert(sizeof(NoAllocFrames) <= 4000, "frame table must fit the kernel parameter space");

__global__ void k_noalloc_frames(const NoAllocFrames p, FrameHost *fh, int *nk, unsigned *status) {
  for (int f = threadIdx.x; f < p.nf; f += blockDim.x) {
    fh[f] = p.fh[f];
    nk[3 * f + 0] = p.nk[f][0];
    nk[3 * f + 1] = p.nk[f][1];
    nk[3 * f + 2] = p.nk[f][2];
  }
  if (threadIdx.x == 0) status[0] = 0u;
}

// Device address of the scratch array in the calling thread's current CUDA
// context.  A symbol's device address belongs to a context, not to a device
// ordinal: after cudaDeviceReset, or with another driver-API context current,
// an address cached per ordinal would be stale.  So the cache is keyed by the
// context's unique id (cuCtxGetId; ids are never reused within a process,
// unlike context handles), and the first call in each context resolves the
// address with cudaGetSymbolAddress (which may load the module into that
// context).  The two driver entry points come through the runtime, so the
// library needs no link to the driver library.
using PfnCtxGetCurrent = CUresult (*)(CUcontext *);
using PfnCtxGetId = CUresult (*)(CUcontext, unsigned long long *);

int noalloc_scratch(unsigned char **out) {
  static std::mutex mu;
  static PfnCtxGetCurrent get_current = nullptr;
  static PfnCtxGetId get_id = nullptr;
  struct Entry {
    unsigned long long id;
    unsigned char *addr;
  };
  static Entry cache[16] = {};
  static int next = 0;
  std::lock_guard<std::mutex> lock(mu);
  if (!get_current || !get_id) {
    void *f1 = nullptr, *f2 = nullptr;
    cudaDriverEntryPointQueryResult q1 = cudaDriverEntryPointSymbolNotFound, q2 = cudaDriverEntryPointSymbolNotFound;
    SOG_CUDA_TRY(cudaGetDriverEntryPoint("cuCtxGetCurrent", &f1, cudaEnableDefault, &q1));
    SOG_CUDA_TRY(cudaGetDriverEntryPoint("cuCtxGetId", &f2, cudaEnableDefault, &q2));
    if (q1 != cudaDriverEntryPointSuccess || q2 != cudaDriverEntryPointSuccess || !f1 || !f2)
      return fail(SOG_ERR_CUDA, "driver entry points cuCtxGetCurrent / cuCtxGetId unavailable");
    get_current = reinterpret_cast<PfnCtxGetCurrent>(f1);
    get_id = reinterpret_cast<PfnCtxGetId>(f2);
  }
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS) return fail(SOG_ERR_CUDA, "cuCtxGetCurrent failed");
  void *p = nullptr;
  if (!ctx) {
    // no context current yet: the runtime call makes the device's primary
    // context current (and resolves the address in it)
    const cudaError_t e = cudaGetSymbolAddress(&p, g_direct_scratch);
    if (e != cudaSuccess) return fail(SOG_ERR_CUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
    if (get_current(&ctx) != CUDA_SUCCESS || !ctx) return fail(SOG_ERR_CUDA, "no CUDA context current");
  }
  unsigned long long id = 0;
  if (get_id(ctx, &id) != CUDA_SUCCESS) return fail(SOG_ERR_CUDA, "cuCtxGetId failed");
  for (const Entry &e : cache)
    if (e.addr && e.id == id) {
      *out = e.addr;
      return SOG_OK;
    }
  if (!p) {
    const cudaError_t e = cudaGetSymbolAddress(&p, g_direct_scratch);
    if (e != cudaSuccess) return fail(SOG_ERR_CUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
  }
  cache[next] = Entry{id, static_cast<unsigned char *>(p)};
  next = (next + 1) % 16;
  *out = static_cast<unsigned char *>(p);
  return SOG_OK;
}

// Carves 256-byte aligned regions off the scratch array in order.
struct Carve {
  size_t off = 0;
  size_t take(size_t bytes) {
    const size_t at = off;
    off += (bytes + 255) & ~(size_t)255;
    return at;
  }
};

template <typename T>
int direct_noalloc_impl(const sog_direct_args *a, unsigned *status_out, cudaStream_t st) {
  const int nf = a->nframes, nch = a->nchannels, M = a->n_gauss;
  if (nf > kNoAllocFrames) return fail(SOG_ERR_INVALID, "no-alloc direct k-sum: more than 64 frames in one call");
  NoAllocFrames frames;
  std::memset(&frames, 0, sizeof(frames));
  frames.nf = nf;
  int64_t kmax = 1, maxat = 0, slots = 0;
  for (int f = 0; f < nf; ++f) {
    for (int c = 0; c < 3; ++c) {
      if (a->nk[3 * f + c] < 0 || a->nk[3 * f + c] > 4096) return fail(SOG_ERR_INVALID, "nk out of range");
      frames.nk[f][c] = a->nk[3 * f + c];
    }
    const int64_t nbox = (int64_t)(a->nk[3 * f] + 1) * (2 * a->nk[3 * f + 1] + 1) * (2 * a->nk[3 * f + 2] + 1);
    kmax = std::max(kmax, nbox);
    maxat = std::max<int64_t>(maxat, a->atom_count[f]);
    frames.fh[f].atom_begin = a->atom_begin[f];
    frames.fh[f].natoms = a->atom_count[f];
    frames.fh[f].slot_base = slots;
    frames.fh[f].k_sq_max = a->k_sq_max[f];
    slots += a->atom_count[f];
  }
  if (kmax > ((int64_t)1 << 31)) return fail(SOG_ERR_INVALID, "mode box too large");
  const unsigned kb = nblk(kmax, kDirThreads);
  const int nx_acc = 4 * M + 13;
  const bool want_grad = a->grad_amp || a->grad_bw2;
  const bool want_vir = a->virial != nullptr;
  const bool want_x = want_grad || want_vir;
  const int qs = (int)std::max<int64_t>(1, std::min<int64_t>(256, (maxat + 16383) / 16384));
  const size_t d8 = sizeof(double);
  Carve cv;
  const size_t o_fh = cv.take(sizeof(FrameHost) * nf);
  const size_t o_nk = cv.take(sizeof(int) * 3 * nf);
  const size_t o_geom = cv.take(sizeof(FrameGeom) * nf);
  const size_t o_status = cv.take(16);
  const size_t o_modes = cv.take(d8 * 4 * kmax * nf);
  const size_t o_sfac = cv.take(d8 * 2 * kmax * nf * nch);
  const size_t o_part = cv.take(d8 * 2 * kb * nf * nch);
  const size_t o_partx = cv.take(want_x ? d8 * nx_acc * kb * nf * nch : 0);
  const size_t o_redE = cv.take(d8 * 2 * nf * nch);
  const size_t o_redX = cv.take(d8 * nx_acc * nf * nch);
  const size_t o_fscal = cv.take(d8 * 4 * nf);
  const size_t o_qsum = cv.take(d8 * 2 * nf * nch);
  const size_t o_qpart = cv.take(d8 * 2 * nf * nch * qs);
  const size_t o_tmp = cv.take(d8 * std::max(reduce_tmp_elems(nf, nch, kb, 2), reduce_tmp_elems(nf, nch, kb, nx_acc)));
  if (cv.off > kNoAllocBytes)
    return fail(SOG_ERR_INVALID, "no-alloc direct k-sum: the call needs " + std::to_string(cv.off) +
                                     " bytes of scratch, the fixed array holds " + std::to_string(kNoAllocBytes) +
                                     " (fewer modes, channels or frames per call, or sog_direct_forward)");
  unsigned char *s = nullptr;
  int rc = noalloc_scratch(&s);
  if (rc != SOG_OK) return rc;
  FrameHost *fhd = reinterpret_cast<FrameHost *>(s + o_fh);
  int *nkd = reinterpret_cast<int *>(s + o_nk);
  FrameGeom *geom = reinterpret_cast<FrameGeom *>(s + o_geom);
  // the caller's status word when given (cleared by the first kernel, then
  // or-ed by every kernel of the call), else a word of the scratch
  unsigned *status = status_out ? status_out : reinterpret_cast<unsigned *>(s + o_status);
  double *qsum = reinterpret_cast<double *>(s + o_qsum);
  double *qpart = reinterpret_cast<double *>(s + o_qpart);
  double *tmp = reinterpret_cast<double *>(s + o_tmp);

  k_noalloc_frames<<<1, 64, 0, st>>>(frames, fhd, nkd, status);
  count_launch();
  k_frame_setup<T><<<nblk(nf, 128), 128, 0, st>>>((const T *)a->cells, fhd, geom, nf, SOG_KCONV_PHYSICAL, 1, 1, 1,
                                                  status);
  count_launch();
  k_qsums<T><<<dim3(nf, nch, qs), 256, 0, st>>>((const T *)a->charges, nch, geom, qpart,
                                                (const T *)a->positions, status);
  k_reduce_parts<<<dim3(nf, nch, 1), 256, 0, st>>>(qpart, nf, nch, qs, 2, 2, qsum);
  count_launch();
  count_launch();
  DirArgs da;
  da.geom = geom;
  da.nk = nkd;
  da.kmax_modes = kmax;
  da.nch = nch;
  da.M = M;
  da.kvec = reinterpret_cast<double *>(s + o_modes);
  da.sfac = reinterpret_cast<double *>(s + o_sfac);
  da.part = reinterpret_cast<double *>(s + o_part);
  da.partx = want_x ? reinterpret_cast<double *>(s + o_partx) : nullptr;
  da.nx_acc = nx_acc;
  double *redE = reinterpret_cast<double *>(s + o_redE);
  double *redX = reinterpret_cast<double *>(s + o_redX);
  double *fscal = reinterpret_cast<double *>(s + o_fscal);
  k_direct_sfac<T><<<dim3(kb, nf), kDirThreads, 0, st>>>(da, (const T *)a->positions, (const T *)a->charges,
                                                         (const T *)a->amp, (const T *)a->bw2);
  count_launch();
  if (want_x) {
    k_direct_extra<T><<<dim3(kb, nf, nch), kDirThreads, 0, st>>>(da, (const T *)a->amp, (const T *)a->bw2,
                                                                 want_grad, want_vir);
    count_launch();
  }
  if ((a->forces || a->potential) && maxat > 0) {
    // the launch shapes of sog_direct_forward: one warp per frame of at most 32 atoms
    if (maxat <= 32)
      k_direct_atoms<T, 32><<<dim3(1, nf), 32, 0, st>>>(da, (const T *)a->positions, (const T *)a->charges,
                                                        a->norm_factor, (T *)a->forces, (T *)a->potential);
    else
      k_direct_atoms<T><<<dim3(nblk(maxat, 128), nf), 128, 0, st>>>(da, (const T *)a->positions,
                                                                    (const T *)a->charges, a->norm_factor,
                                                                    (T *)a->forces, (T *)a->potential);
    count_launch();
  }
  reduce_parts(da.part, nf, nch, kb, 2, 2, redE, tmp, st);
  count_launch();
  if (reduce_split(kb) > 1) count_launch();
  if (want_x) {
    reduce_parts(da.partx, nf, nch, kb, nx_acc, nx_acc, redX, tmp, st);
    count_launch();
    if (reduce_split(kb) > 1) count_launch();
  }
  FinalArgs fa;
  std::memset(&fa, 0, sizeof(fa));
  fa.geom = geom;
  fa.redE = redE;
  fa.redX = redX;
  fa.qsum = qsum;
  fa.amp = a->amp;
  fa.bw2 = a->bw2;
  fa.M = M; fa.nch = nch; fa.nx = 1; fa.ny = 1; fa.nz = 1;
  fa.norm = a->norm_factor;
  fa.self_coeff = a->self_coeff;
  fa.lambda = a->charge_neutral_lambda;
  fa.remove_self = a->remove_self;
  fa.k0 = a->k0_correction;
  fa.want_grad = want_grad;
  fa.want_vir = want_vir;
  fa.direct = 1;
  fa.energy = a->energy;
  fa.grad_amp = a->grad_amp;
  fa.grad_bw2 = a->grad_bw2;
  fa.virial = a->virial;
  fa.fscal = fscal;
  k_finalize_frames<T><<<nblk(nf, 64), 64, 0, st>>>(fa, nf);
  count_launch();
  if (a->potential && maxat > 0) {
    k_finalize_atoms<T><<<dim3(nblk(maxat, 256), nf), 256, 0, st>>>(
        geom, fscal, qsum, (const T *)a->charges, (T *)a->potential, nch, a->norm_factor, a->self_coeff,
        a->charge_neutral_lambda, a->remove_self, a->k0_correction);
    count_launch();
  }
  SOG_CUDA_TRY(cudaGetLastError());
  return SOG_OK;
}

}  // namespace
}  // namespace sogb

extern "C" int sog_direct_forward_noalloc(int dtype, const sog_direct_args *a, unsigned int *status,
                                          void *stream) {
  if (!a) return fail(SOG_ERR_INVALID, "null argument");
  if (dtype != SOG_DTYPE_F64 && dtype != SOG_DTYPE_F32) return fail(SOG_ERR_INVALID, "bad dtype");
  if (a->nframes <= 0) return SOG_OK;
  if (!a->atom_begin || !a->atom_count || !a->nk || !a->k_sq_max || !a->positions || !a->charges ||
      !a->cells || !a->amp || !a->bw2)
    return fail(SOG_ERR_INVALID, "missing input array");
  if (a->nchannels < 1 || a->nchannels > kMaxCh)
    return fail(SOG_ERR_UNSUPPORTED, "direct k-sum supports 1..8 charge channels");
  if (a->n_gauss < 1 || a->n_gauss > kMaxGauss) return fail(SOG_ERR_INVALID, "n_gauss must be in [1, 64]");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == SOG_DTYPE_F64) return direct_noalloc_impl<double>(a, status, st);
  return direct_noalloc_impl<float>(a, status, st);
}
