// Real-space pair sum of non-periodic frames (cell=None or a singular cell):
// compute_potential_realspace, src/sog/module/gaussian.py:822-845, with the
// per-frame penalty of gaussian.py:795-798 and explicit derivatives (the
// reference takes forces, dE/dq and dE/d(amp, bw2) by autograd).
//
//   E_f = norm * ( 1/2 sum_{i != j in f} (q_i . q_j) K(r_ij^2)
//                  + [!remove_self] 1/2 sum_i |q_i|^2 sum_m amp_m )
//         + lambda * sum_c mean_c(q)^2,        K(r^2) = sum_m amp_m e^{-r^2 / (2 bw2_m)}
//
// Work is split into tiles of 32 atoms i x a range of partner atoms j of the
// same frame.  A 256-thread block stages 256 partners at a time in shared
// memory; each warp takes every eighth partner, so the 32 lanes of a warp read
// the same partner (a broadcast) and each lane owns one atom i.  Every thread
// sums its whole row (no atomics): forces, the potential and the per-atom
// energy come out in a fixed order, so results are bit-identical from run to
// run.  Large frames split the partner range over several tiles whose partial
// rows a second kernel adds in order.
//   k_rs_pairs    forces, potential, per-atom energy (or partial rows)
//   k_rs_combine  ordered sum of partial rows (frames split over tiles)
//   k_rs_grad     dE/d(amp, bw2) partials, 8 Gaussian terms per block row
//   k_rs_frames   per-frame energy, parameter gradients, penalty terms
#include <algorithm>
#include <cstring>
#include <vector>

#include "plan.hpp"

namespace sogb {
namespace {

constexpr int kRsI = 32;        // atoms i per tile (one per lane)
constexpr int kRsLanes = 8;     // warps per block, each a stride-8 share of the partners
constexpr int kRsThreads = kRsI * kRsLanes;
constexpr int kRsStage = 256;   // partners staged in shared memory at a time
constexpr int kRsCh = 8;        // charge channels
constexpr int kRsMChunk = 8;    // Gaussian terms per row of the gradient kernel
constexpr int kRsChunkMin = 1024;  // smallest partner range of a split tile
constexpr int kRsMaxSplit = 16;

struct RsFrame {
  int64_t atom_begin;
  int64_t prow;      // first partial row (split frames)
  int32_t natoms;
  int32_t nsplit;    // partner ranges the frame's rows are split into
  int32_t tile_begin;
  int32_t ntiles;
};

struct RsTile {
  int32_t frame;
  int32_t i0;        // first atom i (frame-relative)
  int32_t j0, j1;    // partner range [j0, j1) (frame-relative)
  int32_t split;     // index of the partner range
  int32_t pad[3];
};

struct RsCombineTile {
  int32_t frame;
  int32_t i0;
};

template <typename T>
struct RsArgs {
  const RsFrame *frames;
  const RsTile *tiles;
  const T *pos, *q, *amp, *bw2;
  int nch, M;
  double norm;
  int remove_self;
  T *forces, *pot;
  double *eatom;     // [N] unscaled per-atom energy 1/2 sum_c q_ic p_ic
  double *part;      // [rows][3 + nch] partial force / potential rows
};

// Gaussian-term tables in shared memory: -1/(2 bw2), amp, amp / bw2.
template <typename CT>
struct RsParams {
  CT nh[kMaxGauss], a[kMaxGauss], ad[kMaxGauss];
};

template <typename T, typename CT>
__device__ __forceinline__ void load_params(RsParams<CT> &p, const T *amp, const T *bw2, int M) {
  for (int m = threadIdx.x; m < M; m += blockDim.x) {
    const CT b = (CT)bw2[m], a = (CT)amp[m];
    p.nh[m] = (CT)(-0.5) / b;
    p.a[m] = a;
    p.ad[m] = a / b;
  }
}

__device__ __forceinline__ double rs_exp(double x) { return exp(x); }
__device__ __forceinline__ float rs_exp(float x) { return expf(x); }

template <typename CT, int NCH>
struct RsStage {
  CT x[kRsStage], y[kRsStage], z[kRsStage];
  CT q[NCH][kRsStage];
};

// NCH: channel capacity of the instantiation (nch <= NCH), so a one-channel
// call keeps one charge and one potential accumulator per thread.
template <typename T, int NCH>
__global__ void __launch_bounds__(kRsThreads, 2) k_rs_pairs(RsArgs<T> a) {
  using CT = T;
  __shared__ RsParams<CT> prm;
  __shared__ union {
    RsStage<CT, NCH> st;
    double red[kRsLanes][kRsI][3 + NCH];
  } sm;
  const RsTile t = a.tiles[blockIdx.x];
  const RsFrame fr = a.frames[t.frame];
  load_params(prm, a.amp, a.bw2, a.M);
  const int il = threadIdx.x & (kRsI - 1), jl = threadIdx.x / kRsI;
  const int i = t.i0 + il;
  const bool own = i < fr.natoms;
  const int64_t ai = fr.atom_begin + (own ? i : 0);
  const int nch = a.nch, M = a.M;
  CT xi = 0, yi = 0, zi = 0, qi[NCH];
  if (own) {
    xi = a.pos[ai * 3 + 0];
    yi = a.pos[ai * 3 + 1];
    zi = a.pos[ai * 3 + 2];
  }
#pragma unroll
  for (int c = 0; c < NCH; ++c) qi[c] = (own && c < nch) ? a.q[ai * nch + c] : (CT)0;
  double fx = 0, fy = 0, fz = 0, pc[NCH];
#pragma unroll
  for (int c = 0; c < NCH; ++c) pc[c] = 0.0;
  for (int jb = t.j0; jb < t.j1; jb += kRsStage) {
    __syncthreads();
    const int jj = jb + threadIdx.x;
    if (jj < t.j1) {
      const int64_t aj = fr.atom_begin + jj;
      sm.st.x[threadIdx.x] = a.pos[aj * 3 + 0];
      sm.st.y[threadIdx.x] = a.pos[aj * 3 + 1];
      sm.st.z[threadIdx.x] = a.pos[aj * 3 + 2];
#pragma unroll
      for (int c = 0; c < NCH; ++c)
        if (c < nch) sm.st.q[c][threadIdx.x] = a.q[aj * nch + c];
    }
    __syncthreads();
    const int cnt = min(kRsStage, t.j1 - jb);
    if (!own) continue;
    for (int k = jl; k < cnt; k += kRsLanes) {
      if (jb + k == i) continue;
      const CT dx = xi - sm.st.x[k], dy = yi - sm.st.y[k], dz = zi - sm.st.z[k];
      const CT r2 = dx * dx + dy * dy + dz * dz;
      CT K = 0, Kd = 0;
#pragma unroll 4
      for (int m = 0; m < M; ++m) {
        const CT e = rs_exp(r2 * prm.nh[m]);
        K += prm.a[m] * e;
        Kd += prm.ad[m] * e;
      }
      CT qq = 0;
#pragma unroll
      for (int c = 0; c < NCH; ++c)
        if (c < nch) {
          const CT qj = sm.st.q[c][k];
          qq += qi[c] * qj;
          pc[c] += (double)(K * qj);
        }
      const double s = (double)(qq * Kd);
      fx += s * (double)dx;
      fy += s * (double)dy;
      fz += s * (double)dz;
    }
  }
  __syncthreads();
  sm.red[jl][il][0] = fx;
  sm.red[jl][il][1] = fy;
  sm.red[jl][il][2] = fz;
#pragma unroll
  for (int c = 0; c < NCH; ++c)
    if (c < nch) sm.red[jl][il][3 + c] = pc[c];
  __syncthreads();
  if (jl != 0 || !own) return;
  double acc[3 + NCH];
#pragma unroll
  for (int w = 0; w < 3 + NCH; ++w) acc[w] = 0.0;
  for (int l = 0; l < kRsLanes; ++l) {
#pragma unroll
    for (int w = 0; w < 3 + NCH; ++w)
      if (w < 3 + nch) acc[w] += sm.red[l][il][w];
  }
  if (fr.nsplit > 1) {
    double *row = a.part + (fr.prow + (int64_t)t.split * fr.natoms + i) * (3 + nch);
#pragma unroll
    for (int w = 0; w < 3 + NCH; ++w)
      if (w < 3 + nch) row[w] = acc[w];
    return;
  }
  double asum = 0.0;
  for (int m = 0; m < M; ++m) asum += (double)prm.a[m];
  double e = 0.0;
#pragma unroll
  for (int c = 0; c < NCH; ++c)
    if (c < nch) e += (double)qi[c] * acc[3 + c];
  a.eatom[ai] = 0.5 * e;
  if (a.forces)
#pragma unroll
    for (int d = 0; d < 3; ++d) a.forces[ai * 3 + d] = (T)(a.norm * acc[d]);
  if (a.pot)
#pragma unroll
    for (int c = 0; c < NCH; ++c)
      if (c < nch)
        a.pot[ai * nch + c] = (T)(a.norm * (acc[3 + c] + (a.remove_self ? 0.0 : (double)qi[c] * asum)));
}

template <typename T>
__global__ void __launch_bounds__(256) k_rs_combine(RsArgs<T> a, const RsCombineTile *ct) {
  const RsCombineTile t = ct[blockIdx.x];
  const RsFrame fr = a.frames[t.frame];
  const int i = t.i0 + threadIdx.x;
  if (i >= fr.natoms) return;
  const int nch = a.nch, W = 3 + nch;
  const int64_t ai = fr.atom_begin + i;
  double acc[3 + kRsCh];
#pragma unroll
  for (int w = 0; w < 3 + kRsCh; ++w) acc[w] = 0.0;
  for (int s = 0; s < fr.nsplit; ++s) {
    const double *row = a.part + (fr.prow + (int64_t)s * fr.natoms + i) * W;
#pragma unroll
    for (int w = 0; w < 3 + kRsCh; ++w)
      if (w < W) acc[w] += row[w];
  }
  double asum = 0.0;
  for (int m = 0; m < a.M; ++m) asum += (double)a.amp[m];
  double e = 0.0;
#pragma unroll
  for (int c = 0; c < kRsCh; ++c)
    if (c < nch) e += (double)a.q[ai * nch + c] * acc[3 + c];
  a.eatom[ai] = 0.5 * e;
  if (a.forces)
#pragma unroll
    for (int d = 0; d < 3; ++d) a.forces[ai * 3 + d] = (T)(a.norm * acc[d]);
  if (a.pot)
#pragma unroll
    for (int c = 0; c < kRsCh; ++c)
      if (c < nch)
        a.pot[ai * nch + c] =
            (T)(a.norm * (acc[3 + c] + (a.remove_self ? 0.0 : (double)a.q[ai * nch + c] * asum)));
}

// Deterministic block sum of V values per thread (xor-shuffle tree within a
// warp, then the warps in order); the result is valid in thread 0.
template <int V>
__device__ __forceinline__ void block_sum(double (&v)[V], double (*sh)[V]) {
#pragma unroll
  for (int k = 0; k < V; ++k)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v[k] += __shfl_xor_sync(0xffffffffu, v[k], o);
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if ((threadIdx.x & 31) == 0)
#pragma unroll
    for (int k = 0; k < V; ++k) sh[w][k] = v[k];
  __syncthreads();
  if (threadIdx.x == 0)
    for (int k = 0; k < V; ++k) {
      double s = 0.0;
      for (int u = 0; u < nw; ++u) s += sh[u][k];
      v[k] = s;
    }
}

// Per tile and chunk of 8 Gaussian terms: sum over the tile's pairs of
// (q_i . q_j) e_m and (q_i . q_j) e_m r^2.
template <typename T, int NCH>
__global__ void __launch_bounds__(kRsThreads, 2) k_rs_grad(RsArgs<T> a, double *gpart) {
  using CT = T;
  __shared__ RsParams<CT> prm;
  __shared__ RsStage<CT, NCH> st;
  __shared__ double red[kRsThreads / 32][2 * kRsMChunk];
  const RsTile t = a.tiles[blockIdx.x];
  const RsFrame fr = a.frames[t.frame];
  load_params(prm, a.amp, a.bw2, a.M);
  const int m0 = blockIdx.y * kRsMChunk;
  const int mc = min(kRsMChunk, a.M - m0);
  const int il = threadIdx.x & (kRsI - 1), jl = threadIdx.x / kRsI;
  const int i = t.i0 + il;
  const bool own = i < fr.natoms;
  const int64_t ai = fr.atom_begin + (own ? i : 0);
  const int nch = a.nch;
  CT xi = 0, yi = 0, zi = 0, qi[NCH];
  if (own) {
    xi = a.pos[ai * 3 + 0];
    yi = a.pos[ai * 3 + 1];
    zi = a.pos[ai * 3 + 2];
  }
#pragma unroll
  for (int c = 0; c < NCH; ++c) qi[c] = (own && c < nch) ? a.q[ai * nch + c] : (CT)0;
  double v[2 * kRsMChunk];
#pragma unroll
  for (int k = 0; k < 2 * kRsMChunk; ++k) v[k] = 0.0;
  for (int jb = t.j0; jb < t.j1; jb += kRsStage) {
    __syncthreads();
    const int jj = jb + threadIdx.x;
    if (jj < t.j1) {
      const int64_t aj = fr.atom_begin + jj;
      st.x[threadIdx.x] = a.pos[aj * 3 + 0];
      st.y[threadIdx.x] = a.pos[aj * 3 + 1];
      st.z[threadIdx.x] = a.pos[aj * 3 + 2];
#pragma unroll
      for (int c = 0; c < NCH; ++c)
        if (c < nch) st.q[c][threadIdx.x] = a.q[aj * nch + c];
    }
    __syncthreads();
    const int cnt = min(kRsStage, t.j1 - jb);
    if (!own) continue;
    for (int k = jl; k < cnt; k += kRsLanes) {
      if (jb + k == i) continue;
      const CT dx = xi - st.x[k], dy = yi - st.y[k], dz = zi - st.z[k];
      const CT r2 = dx * dx + dy * dy + dz * dz;
      CT qq = 0;
#pragma unroll
      for (int c = 0; c < NCH; ++c)
        if (c < nch) qq += qi[c] * st.q[c][k];
#pragma unroll
      for (int m = 0; m < kRsMChunk; ++m)
        if (m < mc) {
          const CT e = qq * rs_exp(r2 * prm.nh[m0 + m]);
          v[m] += (double)e;
          v[kRsMChunk + m] += (double)(e * r2);
        }
    }
  }
  block_sum<2 * kRsMChunk>(v, red);
  if (threadIdx.x == 0) {
    double *o = gpart + ((int64_t)blockIdx.x * gridDim.y + blockIdx.y) * (2 * kRsMChunk);
    for (int k = 0; k < 2 * kRsMChunk; ++k) o[k] = v[k];
  }
}

// One block per frame: energy, parameter gradients and penalty terms.
template <typename T>
__global__ void __launch_bounds__(256) k_rs_frames(RsArgs<T> a, const double *gpart, int nmc, double lambda,
                                                  T *energy, T *gamp, T *gbw2) {
  __shared__ double sh[8][2 + kRsCh];
  __shared__ double qmean[kRsCh];
  const int f = blockIdx.x;
  const RsFrame fr = a.frames[f];
  const int nch = a.nch;
  double v[2 + kRsCh];  // sum e_i, sum |q_i|^2, sum_i q_ic
#pragma unroll
  for (int k = 0; k < 2 + kRsCh; ++k) v[k] = 0.0;
  for (int i = threadIdx.x; i < fr.natoms; i += blockDim.x) {
    const int64_t ai = fr.atom_begin + i;
    v[0] += a.eatom[ai];
#pragma unroll
    for (int c = 0; c < kRsCh; ++c)
      if (c < nch) {
        const double qc = (double)a.q[ai * nch + c];
        v[1] += qc * qc;
        v[2 + c] += qc;
      }
  }
  block_sum<2 + kRsCh>(v, sh);
  double asum = 0.0;
  for (int m = 0; m < a.M; ++m) asum += (double)a.amp[m];
  const bool pen = lambda > 0.0 && fr.natoms > 0;
  if (threadIdx.x == 0) {
    double e = a.norm * (v[0] + (a.remove_self ? 0.0 : 0.5 * v[1] * asum));
#pragma unroll
    for (int c = 0; c < kRsCh; ++c)
      if (c < nch) {
        const double mean = fr.natoms > 0 ? v[2 + c] / fr.natoms : 0.0;
        qmean[c] = mean;
        if (pen) e += lambda * mean * mean;
      }
    energy[f] = (T)e;
    sh[0][0] = v[1];
  }
  __syncthreads();
  if (gamp || gbw2) {
    const double qsq = sh[0][0];
    for (int m = threadIdx.x; m < a.M; m += blockDim.x) {
      const int mc = m / kRsMChunk, mm = m % kRsMChunk;
      double se = 0.0, ser = 0.0;
      for (int t = 0; t < fr.ntiles; ++t) {
        const double *o = gpart + ((int64_t)(fr.tile_begin + t) * nmc + mc) * (2 * kRsMChunk);
        se += o[mm];
        ser += o[kRsMChunk + mm];
      }
      const double bw = (double)a.bw2[m];
      if (gamp) gamp[(int64_t)f * a.M + m] = (T)(a.norm * (0.5 * se + (a.remove_self ? 0.0 : 0.5 * qsq)));
      if (gbw2) gbw2[(int64_t)f * a.M + m] = (T)(a.norm * (double)a.amp[m] * ser / (4.0 * bw * bw));
    }
  }
  if (pen && a.pot)
    for (int i = threadIdx.x; i < fr.natoms; i += blockDim.x) {
      const int64_t ai = fr.atom_begin + i;
      for (int c = 0; c < nch; ++c)
        a.pot[ai * nch + c] = (T)((double)a.pot[ai * nch + c] + 2.0 * lambda * qmean[c] / fr.natoms);
    }
}

inline void after(Tracer *tr, cudaStream_t st, const char *name) {
  count_launch();
  if (tr) tr->mark(st, name);
}

// Tiles of one call: each frame's atoms in rows of 32, each row's partners in
// nsplit ranges (multiples of the staging width) when the frame is large and
// the call has too few rows to fill the GPU.
struct RsLayout {
  std::vector<RsFrame> frames;
  std::vector<RsTile> tiles;
  std::vector<RsCombineTile> combine;
  int64_t rows = 0;     // partial rows
  int64_t natoms_end = 0;
};

int rs_layout(const sog_realspace_args *a, int sm_count, RsLayout &L, bool allow_split = true) {
  const int nf = a->nframes;
  L.frames.resize(nf);
  int64_t itiles = 0;
  for (int f = 0; f < nf; ++f) {
    if (a->atom_count[f] < 0 || a->atom_count[f] > ((int64_t)1 << 30) || a->atom_begin[f] < 0)
      return fail(SOG_ERR_INVALID, "atom range of a frame out of bounds");
    itiles += (a->atom_count[f] + kRsI - 1) / kRsI;
    L.natoms_end = std::max(L.natoms_end, a->atom_begin[f] + a->atom_count[f]);
  }
  const int64_t target = (int64_t)sm_count * 2048 / kRsThreads * 4;  // about four waves
  const int64_t want = std::max<int64_t>(1, (target + std::max<int64_t>(itiles, 1) - 1) /
                                                std::max<int64_t>(itiles, 1));
  for (int f = 0; f < nf; ++f) {
    const int n = (int)a->atom_count[f];
    RsFrame &F = L.frames[f];
    F.atom_begin = a->atom_begin[f];
    F.natoms = n;
    const int64_t cap = std::max<int64_t>(1, n / kRsChunkMin);
    int ns = allow_split ? (int)std::min<int64_t>(std::min<int64_t>(want, cap), kRsMaxSplit) : 1;
    int chunk = n;
    if (ns > 1) {
      chunk = (n + ns - 1) / ns;
      chunk = (chunk + kRsStage - 1) / kRsStage * kRsStage;
      ns = (n + chunk - 1) / chunk;
    }
    F.nsplit = ns;
    F.prow = ns > 1 ? L.rows : 0;
    if (ns > 1) L.rows += (int64_t)ns * n;
    F.tile_begin = (int)L.tiles.size();
    for (int i0 = 0; i0 < n; i0 += kRsI)
      for (int s = 0; s < ns; ++s) {
        RsTile t{};
        t.frame = f;
        t.i0 = i0;
        t.j0 = s * chunk;
        t.j1 = std::min(n, (s + 1) * chunk);
        t.split = s;
        L.tiles.push_back(t);
      }
    F.ntiles = (int)L.tiles.size() - F.tile_begin;
    if (ns > 1)
      for (int i0 = 0; i0 < n; i0 += 256) L.combine.push_back(RsCombineTile{f, i0});
  }
  if (L.tiles.size() > (size_t)INT32_MAX) return fail(SOG_ERR_INVALID, "too many tiles");
  return SOG_OK;
}

template <typename T>
int realspace_impl(sog_direct *d, const sog_realspace_args *a, cudaStream_t st) {
  const int nf = a->nframes, nch = a->nchannels, M = a->n_gauss;
  int sm_count = 148;
  {
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess)
      cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, dev);
  }
  RsLayout L;
  int rc = rs_layout(a, sm_count, L);
  if (rc != SOG_OK) return rc;
  const size_t bf = sizeof(RsFrame) * nf, bt = sizeof(RsTile) * L.tiles.size(),
               bc = sizeof(RsCombineTile) * L.combine.size();
  const size_t up_bytes = bf + bt + bc;
  if ((rc = d->up.reserve(up_bytes)) != SOG_OK) return rc;
  if ((rc = d->up.wait()) != SOG_OK) return rc;
  std::memcpy(d->up.p, L.frames.data(), bf);
  if (bt) std::memcpy((char *)d->up.p + bf, L.tiles.data(), bt);
  if (bc) std::memcpy((char *)d->up.p + bf + bt, L.combine.data(), bc);
  const bool want_grad = a->grad_amp || a->grad_bw2;
  const int nmc = (M + kRsMChunk - 1) / kRsMChunk;
  if (d->frames_host_dev.reserve(up_bytes) ||
      d->modes.reserve(sizeof(double) * std::max<int64_t>(1, L.natoms_end)) ||
      d->part.reserve(sizeof(double) * std::max<int64_t>(1, L.rows * (3 + nch))) ||
      (want_grad && d->sfac.reserve(sizeof(double) * 2 * kRsMChunk * std::max<size_t>(1, L.tiles.size()) * nmc)))
    return fail(SOG_ERR_NOMEM, "device allocation failed (real space)");
  SOG_CUDA_TRY(cudaMemcpyAsync(d->frames_host_dev.p, d->up.p, up_bytes, cudaMemcpyHostToDevice, st));
  SOG_CUDA_TRY(cudaEventRecord(d->up.done, st));
  d->up.pending = true;
  RsArgs<T> ra;
  ra.frames = d->frames_host_dev.as<RsFrame>();
  ra.tiles = reinterpret_cast<const RsTile *>((const char *)d->frames_host_dev.p + bf);
  ra.pos = (const T *)a->positions;
  ra.q = (const T *)a->charges;
  ra.amp = (const T *)a->amp;
  ra.bw2 = (const T *)a->bw2;
  ra.nch = nch;
  ra.M = M;
  ra.norm = a->norm_factor;
  ra.remove_self = a->remove_self;
  ra.forces = (T *)a->forces;
  ra.pot = (T *)a->potential;
  ra.eatom = d->modes.as<double>();
  ra.part = d->part.as<double>();
  const RsCombineTile *ctd = reinterpret_cast<const RsCombineTile *>((const char *)d->frames_host_dev.p + bf + bt);
  Tracer *tr = &d->tr;
  tr->begin(st);
  const unsigned ntiles = (unsigned)L.tiles.size();
  if (ntiles) {
    if (nch == 1) k_rs_pairs<T, 1><<<ntiles, kRsThreads, 0, st>>>(ra);
    else if (nch == 2) k_rs_pairs<T, 2><<<ntiles, kRsThreads, 0, st>>>(ra);
    else if (nch <= 4) k_rs_pairs<T, 4><<<ntiles, kRsThreads, 0, st>>>(ra);
    else k_rs_pairs<T, kRsCh><<<ntiles, kRsThreads, 0, st>>>(ra);
    after(tr, st, "rs_pairs");
  }
  if (!L.combine.empty()) {
    k_rs_combine<T><<<(unsigned)L.combine.size(), 256, 0, st>>>(ra, ctd);
    after(tr, st, "rs_combine");
  }
  if (want_grad && ntiles) {
    const dim3 g(ntiles, nmc);
    double *gp = d->sfac.as<double>();
    if (nch == 1) k_rs_grad<T, 1><<<g, kRsThreads, 0, st>>>(ra, gp);
    else if (nch == 2) k_rs_grad<T, 2><<<g, kRsThreads, 0, st>>>(ra, gp);
    else if (nch <= 4) k_rs_grad<T, 4><<<g, kRsThreads, 0, st>>>(ra, gp);
    else k_rs_grad<T, kRsCh><<<g, kRsThreads, 0, st>>>(ra, gp);
    after(tr, st, "rs_grad");
  }
  const double lam = a->charge_neutral_lambda > 0.0 ? a->charge_neutral_lambda : 0.0;
  k_rs_frames<T><<<nf, 256, 0, st>>>(ra, want_grad ? d->sfac.as<double>() : nullptr, nmc, lam, (T *)a->energy,
                                     (T *)a->grad_amp, (T *)a->grad_bw2);
  after(tr, st, "rs_frames");
  if (a->virial) SOG_CUDA_TRY(cudaMemsetAsync(a->virial, 0, sizeof(T) * 9 * nf, st));
  SOG_CUDA_TRY(cudaGetLastError());
  return SOG_OK;
}


// ==========================================================================
// Hessian-vector products (double backward) of the pair sum.
// With Q_ij = q_i . q_j, u = r_i - r_j, s = |u|^2, K(s) = sum_m amp_m e_m,
// e_m = exp(-s / 2 bw2_m), K1 = dK/ds, K2 = d2K/ds2, and a direction (a_i on
// the charges, b_i on the positions, c on (amp, bw2)):
//   ds = 2 u.(b_i - b_j),  dK = sum_m c . dK/d(amp_m, bw2_m),  dK1 = d(dK)/ds,
//   (H d)_{q_ic} = norm sum_j [a_jc K + q_jc (K1 ds + dK)]
//   (H d)_{r_i}  = norm sum_j [(a_i.q_j + q_i.a_j) 2u K1
//                             + Q_ij (2u K2 ds + 2 K1 (b_i - b_j) + 2u dK1)]
//   (H d)_{theta_m} = norm/2 sum_{i != j} [(a_i.q_j + q_i.a_j) dK/dtheta_m
//                                          + Q_ij (dK1/dtheta_m ds + d(dK)/dtheta_m)]
// plus the self term (remove_self = 0) and the neutrality penalty, which
// depend on the charges and amp only.
// ==========================================================================
template <typename T>
struct RsHvp {
  const void *dq, *dr, *damp, *dbw2;
  void *oq, *orr, *oamp, *obw2;
};

template <typename T>
__device__ __forceinline__ double rs_dir(const void *p, int64_t i) {
  return p ? (double)static_cast<const T *>(p)[i] : 0.0;
}

template <typename T, int NCH>
__global__ void __launch_bounds__(kRsThreads, 1) k_rs_hvp_pairs(RsArgs<T> a, RsHvp<T> h) {
  __shared__ double s_nh[kMaxGauss], s_a[kMaxGauss], s_ib[kMaxGauss], s_ca[kMaxGauss], s_cb[kMaxGauss];
  __shared__ union {
    struct {
      double x[kRsStage], y[kRsStage], z[kRsStage], bx[kRsStage], by[kRsStage], bz[kRsStage];
      double q[NCH][kRsStage], d[NCH][kRsStage];
    } st;
    double red[kRsLanes][kRsI][3 + NCH];
  } sm;
  const RsTile t = a.tiles[blockIdx.x];
  const RsFrame fr = a.frames[t.frame];
  for (int m = threadIdx.x; m < a.M; m += blockDim.x) {
    const double b = (double)a.bw2[m];
    s_nh[m] = -0.5 / b;
    s_a[m] = (double)a.amp[m];
    s_ib[m] = 1.0 / b;
    s_ca[m] = rs_dir<T>(h.damp, (int64_t)t.frame * a.M + m);
    s_cb[m] = rs_dir<T>(h.dbw2, (int64_t)t.frame * a.M + m);
  }
  const int il = threadIdx.x & (kRsI - 1), jl = threadIdx.x / kRsI;
  const int i = t.i0 + il;
  const bool own = i < fr.natoms;
  const int64_t ai = fr.atom_begin + (own ? i : 0);
  const int nch = a.nch, M = a.M;
  double ri[3] = {0, 0, 0}, bi[3] = {0, 0, 0}, qi[NCH], di[NCH];
  if (own)
    for (int c = 0; c < 3; ++c) {
      ri[c] = (double)a.pos[ai * 3 + c];
      bi[c] = rs_dir<T>(h.dr, ai * 3 + c);
    }
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    qi[c] = (own && c < nch) ? (double)a.q[ai * nch + c] : 0.0;
    di[c] = (own && c < nch) ? rs_dir<T>(h.dq, ai * nch + c) : 0.0;
  }
  double acc[3 + NCH];
#pragma unroll
  for (int w = 0; w < 3 + NCH; ++w) acc[w] = 0.0;
  for (int jb = t.j0; jb < t.j1; jb += kRsStage) {
    __syncthreads();
    const int jj = jb + threadIdx.x;
    if (jj < t.j1) {
      const int64_t aj = fr.atom_begin + jj;
      sm.st.x[threadIdx.x] = (double)a.pos[aj * 3 + 0];
      sm.st.y[threadIdx.x] = (double)a.pos[aj * 3 + 1];
      sm.st.z[threadIdx.x] = (double)a.pos[aj * 3 + 2];
      sm.st.bx[threadIdx.x] = rs_dir<T>(h.dr, aj * 3 + 0);
      sm.st.by[threadIdx.x] = rs_dir<T>(h.dr, aj * 3 + 1);
      sm.st.bz[threadIdx.x] = rs_dir<T>(h.dr, aj * 3 + 2);
#pragma unroll
      for (int c = 0; c < NCH; ++c)
        if (c < nch) {
          sm.st.q[c][threadIdx.x] = (double)a.q[aj * nch + c];
          sm.st.d[c][threadIdx.x] = rs_dir<T>(h.dq, aj * nch + c);
        }
    }
    __syncthreads();
    const int cnt = min(kRsStage, t.j1 - jb);
    if (!own) continue;
    for (int k = jl; k < cnt; k += kRsLanes) {
      if (jb + k == i) continue;
      const double ux = ri[0] - sm.st.x[k], uy = ri[1] - sm.st.y[k], uz = ri[2] - sm.st.z[k];
      const double dbx = bi[0] - sm.st.bx[k], dby = bi[1] - sm.st.by[k], dbz = bi[2] - sm.st.bz[k];
      const double s2 = ux * ux + uy * uy + uz * uz;
      const double ds = 2.0 * (ux * dbx + uy * dby + uz * dbz);
      double K = 0, K1 = 0, K2 = 0, dK = 0, dK1 = 0;
      for (int m = 0; m < M; ++m) {
        const double e = exp(s2 * s_nh[m]);
        const double ib = s_ib[m], am = s_a[m];
        K += am * e;
        K1 += -0.5 * ib * am * e;
        K2 += 0.25 * ib * ib * am * e;
        dK += (s_ca[m] + s_cb[m] * am * 0.5 * s2 * ib * ib) * e;
        dK1 += (-0.5 * ib * s_ca[m] + s_cb[m] * am * (0.5 * ib * ib - 0.25 * s2 * ib * ib * ib)) * e;
      }
      double Q = 0.0, AQ = 0.0;
#pragma unroll
      for (int c = 0; c < NCH; ++c)
        if (c < nch) {
          const double qj = sm.st.q[c][k], dj = sm.st.d[c][k];
          Q += qi[c] * qj;
          AQ += di[c] * qj + qi[c] * dj;
          acc[3 + c] += dj * K + qj * (K1 * ds + dK);
        }
      const double su = 2.0 * (AQ * K1 + Q * (K2 * ds + dK1));
      const double sb = 2.0 * Q * K1;
      acc[0] += su * ux + sb * dbx;
      acc[1] += su * uy + sb * dby;
      acc[2] += su * uz + sb * dbz;
    }
  }
  __syncthreads();
#pragma unroll
  for (int w = 0; w < 3 + NCH; ++w)
    if (w < 3 + nch) sm.red[jl][il][w] = acc[w];
  __syncthreads();
  if (jl != 0 || !own) return;
  double tot[3 + NCH];
#pragma unroll
  for (int w = 0; w < 3 + NCH; ++w) tot[w] = 0.0;
  for (int l = 0; l < kRsLanes; ++l)
#pragma unroll
    for (int w = 0; w < 3 + NCH; ++w)
      if (w < 3 + nch) tot[w] += sm.red[l][il][w];
  T *orr = static_cast<T *>(h.orr), *oq = static_cast<T *>(h.oq);
  for (int d = 0; d < 3; ++d) orr[ai * 3 + d] = (T)(a.norm * tot[d]);
#pragma unroll
  for (int c = 0; c < NCH; ++c)
    if (c < nch) oq[ai * nch + c] = (T)(a.norm * tot[3 + c]);
}

// Parameter rows per tile and chunk of 8 Gaussian terms (ordered pairs; the
// frames kernel halves them).
template <typename T, int NCH>
__global__ void __launch_bounds__(kRsThreads, 2) k_rs_hvp_grad(RsArgs<T> a, RsHvp<T> h, double *gpart) {
  __shared__ double s_nh[kMaxGauss], s_a[kMaxGauss], s_ib[kMaxGauss], s_ca[kMaxGauss], s_cb[kMaxGauss];
  __shared__ struct {
    double x[kRsStage], y[kRsStage], z[kRsStage], bx[kRsStage], by[kRsStage], bz[kRsStage];
    double q[NCH][kRsStage], d[NCH][kRsStage];
  } st;
  __shared__ double red[kRsThreads / 32][2 * kRsMChunk];
  const RsTile t = a.tiles[blockIdx.x];
  const RsFrame fr = a.frames[t.frame];
  for (int m = threadIdx.x; m < a.M; m += blockDim.x) {
    const double b = (double)a.bw2[m];
    s_nh[m] = -0.5 / b;
    s_a[m] = (double)a.amp[m];
    s_ib[m] = 1.0 / b;
    s_ca[m] = rs_dir<T>(h.damp, (int64_t)t.frame * a.M + m);
    s_cb[m] = rs_dir<T>(h.dbw2, (int64_t)t.frame * a.M + m);
  }
  const int m0 = blockIdx.y * kRsMChunk;
  const int mc = min(kRsMChunk, a.M - m0);
  const int il = threadIdx.x & (kRsI - 1), jl = threadIdx.x / kRsI;
  const int i = t.i0 + il;
  const bool own = i < fr.natoms;
  const int64_t ai = fr.atom_begin + (own ? i : 0);
  const int nch = a.nch;
  double ri[3] = {0, 0, 0}, bi[3] = {0, 0, 0}, qi[NCH], di[NCH];
  if (own)
    for (int c = 0; c < 3; ++c) {
      ri[c] = (double)a.pos[ai * 3 + c];
      bi[c] = rs_dir<T>(h.dr, ai * 3 + c);
    }
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    qi[c] = (own && c < nch) ? (double)a.q[ai * nch + c] : 0.0;
    di[c] = (own && c < nch) ? rs_dir<T>(h.dq, ai * nch + c) : 0.0;
  }
  double v[2 * kRsMChunk];
#pragma unroll
  for (int k = 0; k < 2 * kRsMChunk; ++k) v[k] = 0.0;
  for (int jb = t.j0; jb < t.j1; jb += kRsStage) {
    __syncthreads();
    const int jj = jb + threadIdx.x;
    if (jj < t.j1) {
      const int64_t aj = fr.atom_begin + jj;
      st.x[threadIdx.x] = (double)a.pos[aj * 3 + 0];
      st.y[threadIdx.x] = (double)a.pos[aj * 3 + 1];
      st.z[threadIdx.x] = (double)a.pos[aj * 3 + 2];
      st.bx[threadIdx.x] = rs_dir<T>(h.dr, aj * 3 + 0);
      st.by[threadIdx.x] = rs_dir<T>(h.dr, aj * 3 + 1);
      st.bz[threadIdx.x] = rs_dir<T>(h.dr, aj * 3 + 2);
#pragma unroll
      for (int c = 0; c < NCH; ++c)
        if (c < nch) {
          st.q[c][threadIdx.x] = (double)a.q[aj * nch + c];
          st.d[c][threadIdx.x] = rs_dir<T>(h.dq, aj * nch + c);
        }
    }
    __syncthreads();
    const int cnt = min(kRsStage, t.j1 - jb);
    if (!own) continue;
    for (int k = jl; k < cnt; k += kRsLanes) {
      if (jb + k == i) continue;
      const double ux = ri[0] - st.x[k], uy = ri[1] - st.y[k], uz = ri[2] - st.z[k];
      const double s2 = ux * ux + uy * uy + uz * uz;
      const double ds = 2.0 * (ux * (bi[0] - st.bx[k]) + uy * (bi[1] - st.by[k]) + uz * (bi[2] - st.bz[k]));
      double Q = 0.0, AQ = 0.0;
#pragma unroll
      for (int c = 0; c < NCH; ++c)
        if (c < nch) {
          Q += qi[c] * st.q[c][k];
          AQ += di[c] * st.q[c][k] + qi[c] * st.d[c][k];
        }
#pragma unroll
      for (int m = 0; m < kRsMChunk; ++m)
        if (m < mc) {
          const int mm = m0 + m;
          const double e = exp(s2 * s_nh[mm]), ib = s_ib[mm], am = s_a[mm];
          const double g = 0.5 * s2 * ib * ib * e;            // dK/dbw2_m / amp_m
          v[m] += AQ * e + Q * (-0.5 * ib * e * ds + s_cb[mm] * g);
          v[kRsMChunk + m] += AQ * am * g + Q * (am * e * (0.5 * ib * ib - 0.25 * s2 * ib * ib * ib) * ds +
                                                 s_ca[mm] * g +
                                                 s_cb[mm] * am * e * s2 * (0.25 * s2 * ib * ib * ib * ib - ib * ib * ib));
        }
    }
  }
  block_sum<2 * kRsMChunk>(v, red);
  if (threadIdx.x == 0) {
    double *o = gpart + ((int64_t)blockIdx.x * gridDim.y + blockIdx.y) * (2 * kRsMChunk);
    for (int k = 0; k < 2 * kRsMChunk; ++k) o[k] = v[k];
  }
}

// One block per frame: parameter rows, and the self / penalty terms of the charge rows.
template <typename T>
__global__ void __launch_bounds__(256) k_rs_hvp_frames(RsArgs<T> a, RsHvp<T> h, const double *gpart, int nmc,
                                                      double lambda) {
  __shared__ double sh[8][1 + kRsCh];
  __shared__ double s_sum[1 + kRsCh];
  const int f = blockIdx.x;
  const RsFrame fr = a.frames[f];
  const int nch = a.nch, M = a.M;
  double v[1 + kRsCh];   // sum_i q_i . a_i, sum_i a_ic
#pragma unroll
  for (int k = 0; k < 1 + kRsCh; ++k) v[k] = 0.0;
  for (int i = threadIdx.x; i < fr.natoms; i += blockDim.x) {
    const int64_t ai = fr.atom_begin + i;
#pragma unroll
    for (int c = 0; c < kRsCh; ++c)
      if (c < nch) {
        const double dc = rs_dir<T>(h.dq, ai * nch + c);
        v[0] += (double)a.q[ai * nch + c] * dc;
        v[1 + c] += dc;
      }
  }
  block_sum<1 + kRsCh>(v, sh);
  if (threadIdx.x == 0)
    for (int k = 0; k < 1 + kRsCh; ++k) s_sum[k] = v[k];
  __syncthreads();
  const double self = a.remove_self ? 0.0 : 1.0;
  for (int m = threadIdx.x; m < M; m += blockDim.x) {
    const int mc = m / kRsMChunk, mm = m % kRsMChunk;
    double ga = 0.0, gb = 0.0;
    for (int t = 0; t < fr.ntiles; ++t) {
      const double *o = gpart + ((int64_t)(fr.tile_begin + t) * nmc + mc) * (2 * kRsMChunk);
      ga += o[mm];
      gb += o[kRsMChunk + mm];
    }
    ga = a.norm * (0.5 * ga + self * s_sum[0]);
    gb = a.norm * 0.5 * gb;
    static_cast<T *>(h.oamp)[(int64_t)f * M + m] = (T)ga;
    static_cast<T *>(h.obw2)[(int64_t)f * M + m] = (T)gb;
  }
  double asum = 0.0, dA = 0.0;
  for (int m = 0; m < M; ++m) {
    asum += (double)a.amp[m];
    dA += rs_dir<T>(h.damp, (int64_t)f * M + m);
  }
  const bool pen = lambda > 0.0 && fr.natoms > 0;
  T *oq = static_cast<T *>(h.oq);
  for (int i = threadIdx.x; i < fr.natoms; i += blockDim.x) {
    const int64_t ai = fr.atom_begin + i;
    for (int c = 0; c < nch; ++c) {
      const int64_t o = ai * nch + c;
      double val = (double)oq[o];
      val += a.norm * self * (rs_dir<T>(h.dq, o) * asum + (double)a.q[o] * dA);
      if (pen) val += 2.0 * lambda * s_sum[1 + c] / ((double)fr.natoms * fr.natoms);
      oq[o] = (T)val;
    }
  }
}

template <typename T>
int realspace_hvp_impl(sog_direct *d, const sog_realspace_args *a, const sog_hvp_args *hv, cudaStream_t st) {
  const int nf = a->nframes, nch = a->nchannels, M = a->n_gauss;
  RsLayout L;
  int rc = rs_layout(a, 148, L, false);
  if (rc != SOG_OK) return rc;
  const size_t bf = sizeof(RsFrame) * nf, bt = sizeof(RsTile) * L.tiles.size();
  const size_t up_bytes = bf + bt;
  if ((rc = d->up.reserve(up_bytes)) != SOG_OK) return rc;
  if ((rc = d->up.wait()) != SOG_OK) return rc;
  std::memcpy(d->up.p, L.frames.data(), bf);
  if (bt) std::memcpy((char *)d->up.p + bf, L.tiles.data(), bt);
  const int nmc = (M + kRsMChunk - 1) / kRsMChunk;
  if (d->frames_host_dev.reserve(up_bytes) ||
      d->hpart.reserve(sizeof(double) * 2 * kRsMChunk * std::max<size_t>(1, L.tiles.size()) * nmc))
    return fail(SOG_ERR_NOMEM, "device allocation failed (real-space HVP)");
  SOG_CUDA_TRY(cudaMemcpyAsync(d->frames_host_dev.p, d->up.p, up_bytes, cudaMemcpyHostToDevice, st));
  SOG_CUDA_TRY(cudaEventRecord(d->up.done, st));
  d->up.pending = true;
  RsArgs<T> ra;
  std::memset(&ra, 0, sizeof(ra));
  ra.frames = d->frames_host_dev.as<RsFrame>();
  ra.tiles = reinterpret_cast<const RsTile *>((const char *)d->frames_host_dev.p + bf);
  ra.pos = (const T *)a->positions;
  ra.q = (const T *)a->charges;
  ra.amp = (const T *)a->amp;
  ra.bw2 = (const T *)a->bw2;
  ra.nch = nch;
  ra.M = M;
  ra.norm = a->norm_factor;
  ra.remove_self = a->remove_self;
  RsHvp<T> h;
  h.dq = hv->dir_q;
  h.dr = hv->dir_r;
  h.damp = hv->dir_amp;
  h.dbw2 = hv->dir_bw2;
  h.oq = hv->out_q;
  h.orr = hv->out_r;
  h.oamp = hv->out_amp;
  h.obw2 = hv->out_bw2;
  Tracer *tr = &d->tr;
  tr->begin(st);
  const unsigned ntiles = (unsigned)L.tiles.size();
  double *gp = d->hpart.as<double>();
  if (ntiles) {
    if (nch == 1) k_rs_hvp_pairs<T, 1><<<ntiles, kRsThreads, 0, st>>>(ra, h);
    else if (nch == 2) k_rs_hvp_pairs<T, 2><<<ntiles, kRsThreads, 0, st>>>(ra, h);
    else if (nch <= 4) k_rs_hvp_pairs<T, 4><<<ntiles, kRsThreads, 0, st>>>(ra, h);
    else k_rs_hvp_pairs<T, kRsCh><<<ntiles, kRsThreads, 0, st>>>(ra, h);
    after(tr, st, "rs_hvp_pairs");
    const dim3 g(ntiles, nmc);
    if (nch == 1) k_rs_hvp_grad<T, 1><<<g, kRsThreads, 0, st>>>(ra, h, gp);
    else if (nch == 2) k_rs_hvp_grad<T, 2><<<g, kRsThreads, 0, st>>>(ra, h, gp);
    else if (nch <= 4) k_rs_hvp_grad<T, 4><<<g, kRsThreads, 0, st>>>(ra, h, gp);
    else k_rs_hvp_grad<T, kRsCh><<<g, kRsThreads, 0, st>>>(ra, h, gp);
    after(tr, st, "rs_hvp_grad");
  }
  const double lam = a->charge_neutral_lambda > 0.0 ? a->charge_neutral_lambda : 0.0;
  k_rs_hvp_frames<T><<<nf, 256, 0, st>>>(ra, h, gp, nmc, lam);
  after(tr, st, "rs_hvp_frames");
  SOG_CUDA_TRY(cudaGetLastError());
  return SOG_OK;
}
}  // namespace
}  // namespace sogb

using namespace sogb;

extern "C" int sog_realspace_forward(sog_direct *d, const sog_realspace_args *a, void *stream) {
  if (!d || !a) return fail(SOG_ERR_INVALID, "null argument");
  if (a->nframes <= 0) return SOG_OK;
  if (!a->atom_begin || !a->atom_count || !a->positions || !a->charges || !a->amp || !a->bw2 || !a->energy)
    return fail(SOG_ERR_INVALID, "missing input array");
  if (a->nchannels < 1 || a->nchannels > kRsCh)
    return fail(SOG_ERR_UNSUPPORTED, "real-space pair sum supports 1..8 charge channels");
  if (a->n_gauss < 1 || a->n_gauss > kMaxGauss) return fail(SOG_ERR_INVALID, "n_gauss must be in [1, 64]");
  DeviceGuard dg(d->device);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (d->dtype == SOG_DTYPE_F64) return realspace_impl<double>(d, a, st);
  return realspace_impl<float>(d, a, st);
}

extern "C" int sog_realspace_hvp(sog_direct *d, const sog_realspace_args *a, const sog_hvp_args *h, void *stream) {
  if (!d || !a || !h) return fail(SOG_ERR_INVALID, "null argument");
  if (a->nframes <= 0) return SOG_OK;
  if (!a->atom_begin || !a->atom_count || !a->positions || !a->charges || !a->amp || !a->bw2)
    return fail(SOG_ERR_INVALID, "missing input array");
  if (!h->out_q || !h->out_r || !h->out_amp || !h->out_bw2) return fail(SOG_ERR_INVALID, "missing HVP output array");
  if (a->nchannels < 1 || a->nchannels > kRsCh)
    return fail(SOG_ERR_UNSUPPORTED, "real-space pair sum supports 1..8 charge channels");
  if (a->n_gauss < 1 || a->n_gauss > kMaxGauss) return fail(SOG_ERR_INVALID, "n_gauss must be in [1, 64]");
  DeviceGuard dg(d->device);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (d->dtype == SOG_DTYPE_F64) return realspace_hvp_impl<double>(d, a, h, st);
  return realspace_hvp_impl<float>(d, a, h, st);
}
