// Mixed-radix (2,3,4,5,8) Stockham FFT in shared memory, plus the three pass
// kernels of a 3-D real transform on the [nz][ny][nx] mesh:
//   - rows along x: R2C (forward) and C2R (inverse, torch.fft.irfftn
//     semantics: the imaginary parts of the self-conjugate columns are ignored),
//   - strided C2C passes along y and z.
// Each pass reads and writes its array once (HBM-bound); the smem transform
// uses a per-axis table of n-th roots of unity computed on the host in double.
#pragma once
#include "common.cuh"

namespace sogb {

struct RadixPlan {
  int n;
  int nst;
  int r[24];
  // per stage s: n / r[s] and the stride Ns (product of the earlier radices),
  // each with the multiplier of exact division by it for the small indices of
  // a transform, q = umulhi(x, m) for m = floor(2^32 / d) + 1, exact for
  // x < 2^32 / d (Granlund and Montgomery's round-up method)
  int nR[24], Ns[24];
  uint32_t m_nR[24], m_Ns[24];
};

__host__ __device__ __forceinline__ uint32_t fdiv_mul(uint32_t d) {
  return d <= 1 ? 0u : (uint32_t)((((uint64_t)1) << 32) / d + 1);   // 0 marks d == 1
}
__device__ __forceinline__ int fdiv(int x, uint32_t m) { return m ? (int)__umulhi((uint32_t)x, m) : x; }

// DFT of radix R in registers; DIR = -1 forward (e^{-i}), +1 inverse.
template <typename T, int DIR>
__device__ __forceinline__ void dft2(cplx_t<T> *v) {
  cplx_t<T> a = v[0], b = v[1];
  v[0] = cadd(a, b);
  v[1] = csub(a, b);
}

// multiply by -i*DIR... helpers: rot(x) = x * (DIR<0 ? -i : +i)
template <typename T, int DIR>
__device__ __forceinline__ cplx_t<T> rot90(cplx_t<T> x) {
  cplx_t<T> r;
  if (DIR < 0) { r.x = x.y; r.y = -x.x; } else { r.x = -x.y; r.y = x.x; }
  return r;
}

template <typename T, int DIR>
__device__ __forceinline__ void dft4(cplx_t<T> *v) {
  cplx_t<T> a = cadd(v[0], v[2]), b = csub(v[0], v[2]);
  cplx_t<T> c = cadd(v[1], v[3]), d = rot90<T, DIR>(csub(v[1], v[3]));
  v[0] = cadd(a, c);
  v[2] = csub(a, c);
  v[1] = cadd(b, d);
  v[3] = csub(b, d);
}

template <typename T, int DIR>
__device__ __forceinline__ void dft3(cplx_t<T> *v) {
  const T c = T(-0.5);
  const T s = T(0.86602540378443864676372317075294);  // sin(2 pi / 3)
  cplx_t<T> t1 = cadd(v[1], v[2]), t2 = csub(v[1], v[2]);
  cplx_t<T> x0 = cadd(v[0], t1);
  cplx_t<T> a;
  a.x = v[0].x + c * t1.x;
  a.y = v[0].y + c * t1.y;
  // b = s * t2 rotated by -i (forward)
  cplx_t<T> b = rot90<T, DIR>(cmk<cplx_t<T>, T>(s * t2.x, s * t2.y));
  v[0] = x0;
  v[1] = cadd(a, b);
  v[2] = csub(a, b);
}

template <typename T, int DIR>
__device__ __forceinline__ void dft5(cplx_t<T> *v) {
  const T c1 = T(0.30901699437494742410229341718282);   // cos(2 pi/5)
  const T c2 = T(-0.80901699437494742410229341718282);  // cos(4 pi/5)
  const T s1 = T(0.95105651629515357211643933337938);   // sin(2 pi/5)
  const T s2 = T(0.58778525229247312916870595463907);   // sin(4 pi/5)
  cplx_t<T> t1 = cadd(v[1], v[4]), t2 = cadd(v[2], v[3]);
  cplx_t<T> t3 = csub(v[1], v[4]), t4 = csub(v[2], v[3]);
  cplx_t<T> x0 = cadd(v[0], cadd(t1, t2));
  cplx_t<T> a1 = cmk<cplx_t<T>, T>(v[0].x + c1 * t1.x + c2 * t2.x, v[0].y + c1 * t1.y + c2 * t2.y);
  cplx_t<T> a2 = cmk<cplx_t<T>, T>(v[0].x + c2 * t1.x + c1 * t2.x, v[0].y + c2 * t1.y + c1 * t2.y);
  cplx_t<T> b1 = rot90<T, DIR>(cmk<cplx_t<T>, T>(s1 * t3.x + s2 * t4.x, s1 * t3.y + s2 * t4.y));
  cplx_t<T> b2 = rot90<T, DIR>(cmk<cplx_t<T>, T>(s2 * t3.x - s1 * t4.x, s2 * t3.y - s1 * t4.y));
  v[0] = x0;
  v[1] = cadd(a1, b1);
  v[4] = csub(a1, b1);
  v[2] = cadd(a2, b2);
  v[3] = csub(a2, b2);
}

template <typename T, int DIR>
__device__ __forceinline__ void dft8(cplx_t<T> *v) {
  const T h = T(0.70710678118654752440084436210485);  // 1/sqrt(2)
  cplx_t<T> e[4] = {v[0], v[2], v[4], v[6]};
  cplx_t<T> o[4] = {v[1], v[3], v[5], v[7]};
  dft4<T, DIR>(e);
  dft4<T, DIR>(o);
  // twiddles W8^m, W8 = e^{DIR i pi/4}
  cplx_t<T> w1 = cmk<cplx_t<T>, T>(h * (o[1].x - T(DIR) * o[1].y), h * (o[1].y + T(DIR) * o[1].x));
  cplx_t<T> w2 = rot90<T, DIR>(o[2]);
  cplx_t<T> r3 = rot90<T, DIR>(o[3]);
  cplx_t<T> w3 = cmk<cplx_t<T>, T>(h * (r3.x - T(DIR) * r3.y), h * (r3.y + T(DIR) * r3.x));
  v[0] = cadd(e[0], o[0]);
  v[4] = csub(e[0], o[0]);
  v[1] = cadd(e[1], w1);
  v[5] = csub(e[1], w1);
  v[2] = cadd(e[2], w2);
  v[6] = csub(e[2], w2);
  v[3] = cadd(e[3], w3);
  v[7] = csub(e[3], w3);
}

template <typename T, int DIR, int R>
__device__ __forceinline__ void stage_body(const cplx_t<T> *src, cplx_t<T> *dst, int nR, int Ns, uint32_t mNs,
                                           int step, int j, int b, int sj, int sb,
                                           const cplx_t<T> *__restrict__ tw) {
  using C = cplx_t<T>;
  C v[R];
#pragma unroll
  for (int r = 0; r < R; ++r) v[r] = src[(j + r * nR) * sj + b * sb];
  const int jq = Ns > 1 ? fdiv(j, mNs) : j;
  const int k = j - jq * Ns;
  if (Ns > 1) {
#pragma unroll
    for (int r = 1; r < R; ++r) {
      C w = tw[r * k * step];
      if (DIR > 0) w.y = -w.y;
      v[r] = cmul(v[r], w);
    }
  }
  if (R == 2) dft2<T, DIR>(v);
  else if (R == 3) dft3<T, DIR>(v);
  else if (R == 4) dft4<T, DIR>(v);
  else if (R == 5) dft5<T, DIR>(v);
  else dft8<T, DIR>(v);
  const int idxD = jq * Ns * R + k;
#pragma unroll
  for (int r = 0; r < R; ++r) dst[(idxD + r * Ns) * sj + b * sb] = v[r];
}

// `batch` transforms of length rp.n held in smem: element j of transform b at
// a[j*sj + b*sb].  Ping-pongs between a and b; returns the buffer with the
// result.  All threads of the block must call it.
// Column layout (sb == 1, sj = 2^lg_cols >= batch): consecutive threads take
// consecutive transforms of the same element index, so a warp reads
// consecutive words; row layout (sj == 1): consecutive element indices.
// Divisions by the stage constants use the plan's multipliers.
template <typename T, int DIR>
__device__ cplx_t<T> *fft_smem(cplx_t<T> *a, cplx_t<T> *bbuf, const RadixPlan &rp, int batch,
                               int sj, int sb, const cplx_t<T> *__restrict__ tw, int lg_cols = -1,
                               int tws = 1) {
  // tws: stride of the root table (2 when tw holds the roots of twice rp.n)
  cplx_t<T> *src = a, *dst = bbuf;
  for (int s = 0; s < rp.nst; ++s) {
    const int R = rp.r[s], nR = rp.nR[s], Ns = rp.Ns[s];
    const uint32_t mnR = rp.m_nR[s], mNs = rp.m_Ns[s];
    const int step = nR / Ns * tws;   // n / (Ns R), in units of the table
    const int total = lg_cols >= 0 ? (nR << lg_cols) : batch * nR;
    for (int t = threadIdx.x; t < total; t += blockDim.x) {
      int b, j;
      if (lg_cols >= 0) {
        b = t & ((1 << lg_cols) - 1);
        j = t >> lg_cols;
        if (b >= batch) continue;
      } else {
        b = nR > 1 ? fdiv(t, mnR) : t;
        j = t - b * nR;
      }
      switch (R) {
        case 2: stage_body<T, DIR, 2>(src, dst, nR, Ns, mNs, step, j, b, sj, sb, tw); break;
        case 3: stage_body<T, DIR, 3>(src, dst, nR, Ns, mNs, step, j, b, sj, sb, tw); break;
        case 4: stage_body<T, DIR, 4>(src, dst, nR, Ns, mNs, step, j, b, sj, sb, tw); break;
        case 5: stage_body<T, DIR, 5>(src, dst, nR, Ns, mNs, step, j, b, sj, sb, tw); break;
        default: stage_body<T, DIR, 8>(src, dst, nR, Ns, mNs, step, j, b, sj, sb, tw); break;
      }
    }
    __syncthreads();
    cplx_t<T> *tmp = src; src = dst; dst = tmp;
  }
  return src;
}

// Forward R2C along x.  in: nrows rows of nx reals; out: nrows rows of nx/2+1.
template <typename T>
__global__ void k_fft_r2c_x(const T *__restrict__ in, cplx_t<T> *__restrict__ out, int nx,
                            int64_t nrows, int rows_per_cta, RadixPlan rp,
                            const cplx_t<T> *__restrict__ tw) {
  using C = cplx_t<T>;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  C *a = reinterpret_cast<C *>(smem_raw);
  C *b = a + (size_t)rows_per_cta * nx;
  const int64_t row0 = (int64_t)blockIdx.x * rows_per_cta;
  const int nr = (int)min((int64_t)rows_per_cta, nrows - row0);
  const T *src = in + row0 * nx;
  for (int i = threadIdx.x; i < nr * nx; i += blockDim.x) a[i] = cmk<C, T>(src[i], T(0));
  __syncthreads();
  C *res = fft_smem<T, -1>(a, b, rp, nr, 1, nx, tw);
  const int nxh = nx / 2 + 1;
  C *dst = out + row0 * nxh;
  for (int i = threadIdx.x; i < nr * nxh; i += blockDim.x) {
    const int r = i / nxh, x = i - r * nxh;
    dst[i] = res[r * nx + x];
  }
}

// Inverse C2R along x with torch.fft.irfftn semantics (unnormalised).  Input
// rows are field-major, in[((frame*F + f)*nzy + zy)*(nx/2+1) + m]; the output
// is interleaved, out[((frame*nzy + zy)*nx + x)*F + f].  A CTA transforms the
// F fields of `rows_per_cta` consecutive (frame, zy) rows together, so its
// output is one contiguous run of rows_per_cta*nx*F values.  Transform rows
// are nx+1 apart in shared memory.
template <typename T>
__global__ void k_fft_c2r_x(const cplx_t<T> *__restrict__ in, T *__restrict__ out, int nx,
                            int64_t nrows, int rows_per_cta, RadixPlan rp,
                            const cplx_t<T> *__restrict__ tw, int F, int64_t nzy) {
  using C = cplx_t<T>;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int ld = nx + 1;
  C *a = reinterpret_cast<C *>(smem_raw);
  C *b = a + (size_t)rows_per_cta * F * ld;
  const int64_t row0 = (int64_t)blockIdx.x * rows_per_cta;   // (frame, zy) rows
  const int nr = (int)min((int64_t)rows_per_cta, nrows - row0);
  const int nxh = nx / 2 + 1;
  const int nt = nr * F;
  for (int i = threadIdx.x; i < nt * nxh; i += blockDim.x) {
    const int tr = i / nxh, m = i - tr * nxh;      // transform (rl, f), mode m
    const int rl = tr / F, f = tr - rl * F;
    const int64_t row = row0 + rl, frame = row / nzy, zy = row - frame * nzy;
    const C v = in[((frame * F + f) * nzy + zy) * nxh + m];
    C *ar = a + (size_t)tr * ld;
    ar[m] = v;
    if (m >= 1 && m < (nx + 1) / 2) ar[nx - m] = cmk<C, T>(v.x, -v.y);
  }
  __syncthreads();
  C *res = fft_smem<T, +1>(a, b, rp, nt, 1, ld, tw);
  T *dst = out + row0 * nx * F;
  for (int i = threadIdx.x; i < nr * nx * F; i += blockDim.x) {
    const int rl = i / (nx * F), rem = i - rl * nx * F;
    const int x = rem / F, f = rem - x * F;
    dst[i] = res[(size_t)(rl * F + f) * ld + x].x;
  }
}

// Even nx: real rows as length-h complex transforms (h = nx/2), the standard
// packing z[m] = x[2m] + i x[2m+1] with the pre/post twiddle of the
// power-of-two pipelines (fft_pipe.cuh), half the work of a length-nx complex
// transform.  rph is the plan of h; tw the nx-th roots (read with stride 2).
template <typename T>
__global__ void k_fft_r2c_xh(const T *__restrict__ in, cplx_t<T> *__restrict__ out, int nx, int64_t nrows,
                             int rows_per_cta, RadixPlan rph, const cplx_t<T> *__restrict__ tw) {
  using C = cplx_t<T>;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int h = nx / 2, nxh = h + 1;
  C *a = reinterpret_cast<C *>(smem_raw);
  C *b = a + (size_t)rows_per_cta * h;
  const int64_t row0 = (int64_t)blockIdx.x * rows_per_cta;
  const int nr = (int)min((int64_t)rows_per_cta, nrows - row0);
  const C *src = reinterpret_cast<const C *>(in + row0 * nx);   // pairs (x[2m], x[2m+1])
  for (int i = threadIdx.x; i < nr * h; i += blockDim.x) a[i] = src[i];
  __syncthreads();
  C *res = fft_smem<T, -1>(a, b, rph, nr, 1, h, tw, -1, 2);
  C *dst = out + row0 * nxh;
  const uint32_t mh = fdiv_mul((uint32_t)h);
  for (int i = threadIdx.x; i < nr * h; i += blockDim.x) {
    const int r = fdiv(i, mh), k = i - r * h;
    const C za = res[r * h + k];
    const C zb = res[r * h + (k == 0 ? 0 : h - k)];
    const T er = T(0.5) * (za.x + zb.x), ei = T(0.5) * (za.y - zb.y);   // (Z + conj Z')/2
    const T dr = T(0.5) * (za.x - zb.x), di = T(0.5) * (za.y + zb.y);   // (Z - conj Z')/2
    const C w = tw[k];                                                   // W_n^k
    const T pr = w.x * dr - w.y * di, pi = w.x * di + w.y * dr;          // w * d; -i w d below
    dst[r * nxh + k] = cmk<C, T>(er + pi, ei - pr);
    if (k == 0) dst[r * nxh + h] = cmk<C, T>(er - pi, ei + pr);          // k = n/2: W^{n/2} = -1
  }
}

// Even nx inverse: per (frame, zy) row and field, Z[k] = A + i conj(W^k) B
// with A = X[k] + conj X[h-k], B = X[k] - conj X[h-k] (k = 0: the real parts
// of X[0] and X[h] only, torch.fft.irfftn's treatment), inverse length-h
// transform, x[2m] = Re z[m], x[2m+1] = Im z[m]; output interleaved as
// k_fft_c2r_x's.
template <typename T>
__global__ void k_fft_c2r_xh(const cplx_t<T> *__restrict__ in, T *__restrict__ out, int nx, int64_t nrows,
                             int rows_per_cta, RadixPlan rph, const cplx_t<T> *__restrict__ tw, int F,
                             int64_t nzy) {
  using C = cplx_t<T>;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int h = nx / 2, nxh = h + 1, ld = h + 1;
  C *a = reinterpret_cast<C *>(smem_raw);
  C *b = a + (size_t)rows_per_cta * F * ld;
  const int64_t row0 = (int64_t)blockIdx.x * rows_per_cta;   // (frame, zy) rows
  const int nr = (int)min((int64_t)rows_per_cta, nrows - row0);
  const int nt = nr * F;
  // source row of each transform (rl, f): the 64-bit divisions once per row
  __shared__ int64_t srow[256];
  for (int tr = threadIdx.x; tr < nt && tr < 256; tr += blockDim.x) {
    const int rl = tr / F, f = tr - rl * F;
    const int64_t row = row0 + rl, frame = row / nzy, zy = row - frame * nzy;
    srow[tr] = ((frame * F + f) * nzy + zy) * nxh;
  }
  __syncthreads();
  const uint32_t mnxh = fdiv_mul((uint32_t)nxh), mh = fdiv_mul((uint32_t)h);
  const uint32_t mF = fdiv_mul((uint32_t)F), mnxF = fdiv_mul((uint32_t)(nx * F));
  for (int i = threadIdx.x; i < nt * nxh; i += blockDim.x) {
    const int tr = fdiv(i, mnxh), m = i - tr * nxh;
    b[(size_t)tr * ld + m] = in[srow[tr] + m];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < nt * h; i += blockDim.x) {
    const int tr = fdiv(i, mh), k = i - tr * h;
    const C *X = b + (size_t)tr * ld;
    C v;
    if (k == 0) {
      const T x0 = X[0].x, xh = X[h].x;
      v = cmk<C, T>(x0 + xh, x0 - xh);
    } else {
      const C xa = X[k], xb = X[h - k];
      const T Ar = xa.x + xb.x, Ai = xa.y - xb.y;
      const T Br = xa.x - xb.x, Bi = xa.y + xb.y;
      const C w = tw[k];
      const T cr = w.x * Br + w.y * Bi, ci = w.x * Bi - w.y * Br;   // conj(w) * B
      v = cmk<C, T>(Ar - ci, Ai + cr);
    }
    a[(size_t)tr * ld + k] = v;
  }
  __syncthreads();
  C *res = fft_smem<T, +1>(a, b, rph, nt, 1, ld, tw, -1, 2);
  T *dst = out + row0 * nx * F;
  for (int i = threadIdx.x; i < nr * nx * F; i += blockDim.x) {
    const int rl = fdiv(i, mnxF), rem = i - rl * nx * F;
    const int x = fdiv(rem, mF), f = rem - x * F;
    const C z = res[(size_t)(rl * F + f) * ld + (x >> 1)];
    dst[i] = (x & 1) ? z.y : z.x;
  }
}

// C2C along a strided axis: data viewed as [outer][n][inner]; a CTA handles one
// outer index and `ic` (a power of two) consecutive inner columns.
template <typename T, int DIR>
__global__ void k_fft_strided(cplx_t<T> *__restrict__ data, int64_t inner, int64_t outer,
                              int ic, RadixPlan rp, const cplx_t<T> *__restrict__ tw) {
  using C = cplx_t<T>;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int n = rp.n;
  C *a = reinterpret_cast<C *>(smem_raw);
  C *b = a + (size_t)n * ic;
  const int64_t nchunks = (inner + ic - 1) / ic;
  const int64_t o = blockIdx.x / nchunks;
  const int64_t i0 = (blockIdx.x - o * nchunks) * ic;
  const int nic = (int)min((int64_t)ic, inner - i0);
  C *base = data + o * (int64_t)n * inner + i0;
  const int lg = 31 - __clz(ic);
  for (int t = threadIdx.x; t < n * ic; t += blockDim.x) {
    const int j = t >> lg, c = t & (ic - 1);
    if (c < nic) a[t] = base[(int64_t)j * inner + c];
  }
  __syncthreads();
  C *res = fft_smem<T, DIR>(a, b, rp, nic, ic, 1, tw, lg);
  for (int t = threadIdx.x; t < n * ic; t += blockDim.x) {
    const int j = t >> lg, c = t & (ic - 1);
    if (c < nic) base[(int64_t)j * inner + c] = res[t];
  }
}

}  // namespace sogb
