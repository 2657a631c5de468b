// Register-resident Stockham FFT for power-of-two lengths (radix 8/4/2).
//
// Each thread of a transform keeps EPT = 8 elements x[t + e*TPT] (TPT = n/8)
// in registers for the whole transform.  In a stage of radix R a thread runs
// 8/R butterflies j = t + u*TPT on its own elements, writes the outputs to
// their Stockham positions in shared memory and, after a barrier, reads back
// x[t + e*TPT] for the next stage.  The first stage takes its inputs straight
// from HBM and the last stage leaves the outputs in registers in natural order
// (thread t holds X[t + e*TPT]), so a pass costs one HBM read, one HBM write and
// (stages - 1) shared-memory exchanges.
#pragma once
#include "fft.cuh"

namespace sogb {

constexpr int kEPT = 8;

inline bool is_pow2(int n) { return n >= 8 && (n & (n - 1)) == 0; }

template <typename T, int DIR, int R>
__device__ __forceinline__ void dftR(cplx_t<T> *a) {
  if (R == 2) dft2<T, DIR>(a);
  else if (R == 4) dft4<T, DIR>(a);
  else dft8<T, DIR>(a);
}

// Shared-memory slot of element i of a transform whose elements are sj slots
// apart.  A quarter warp issues eight 16-byte accesses; column tiles of width
// sj >= 8 put one full row in it and need no padding.  Rows (sj == 1) and
// narrow tiles (PAD) skip one element-row every 8 so that the stride-8
// Stockham writes of a quarter warp fall in distinct banks.
template <bool PAD>
__device__ __forceinline__ int sidx(int i, int sj) { return PAD ? (i + (i >> 3)) * sj : i * sj; }

// One radix-R stage on the registers v; Ns = product of earlier radices.
template <typename T, int DIR, int R, bool PAD>
__device__ __forceinline__ void reg_stage(cplx_t<T> (&v)[kEPT], int t, int TPT, int n, int Ns,
                                          const cplx_t<T> *__restrict__ tw, cplx_t<T> *sbase,
                                          int sj, bool last) {
  constexpr int B = kEPT / R;
#pragma unroll
  for (int u = 0; u < B; ++u) {
    const int j = t + u * TPT;
    const int k = j & (Ns - 1);
    cplx_t<T> a[R];
#pragma unroll
    for (int r = 0; r < R; ++r) a[r] = v[u + r * B];
    if (Ns > 1) {
      const int step = n / (Ns * R);
#pragma unroll
      for (int r = 1; r < R; ++r) {
        cplx_t<T> w = tw[r * k * step];
        if (DIR > 0) w.y = -w.y;
        a[r] = cmul(a[r], w);
      }
    }
    dftR<T, DIR, R>(a);
    if (last) {
      // j < Ns here, so the outputs j + r*Ns = t + (u + r*B)*TPT stay in v
#pragma unroll
      for (int r = 0; r < R; ++r) v[u + r * B] = a[r];
    } else {
      const int idxD = (j / Ns) * Ns * R + k;
#pragma unroll
      for (int r = 0; r < R; ++r) sbase[sidx<PAD>(idxD + r * Ns, sj)] = a[r];
    }
  }
}

// Whole transform; every thread of the block must call it (barriers inside).
template <typename T, int DIR, bool PAD = false>
__device__ __forceinline__ void reg_fft(cplx_t<T> (&v)[kEPT], int t, const RadixPlan &rp,
                                        const cplx_t<T> *__restrict__ tw, cplx_t<T> *sbase, int sj) {
  const int n = rp.n, TPT = n / kEPT;
  int Ns = 1;
  for (int s = 0; s < rp.nst; ++s) {
    const int R = rp.r[s];
    const bool last = s == rp.nst - 1;
    if (R == 8) reg_stage<T, DIR, 8, PAD>(v, t, TPT, n, Ns, tw, sbase, sj, last);
    else if (R == 4) reg_stage<T, DIR, 4, PAD>(v, t, TPT, n, Ns, tw, sbase, sj, last);
    else reg_stage<T, DIR, 2, PAD>(v, t, TPT, n, Ns, tw, sbase, sj, last);
    if (!last) {
      __syncthreads();
#pragma unroll
      for (int e = 0; e < kEPT; ++e) v[e] = sbase[sidx<PAD>(t + e * TPT, sj)];
      __syncthreads();
    }
    Ns *= R;
  }
}

// ---------------------------------------------------------------------------
// Compile-time length n = 2^L: radix 8 stages, then one radix 4 or 2 stage;
// stage s has Ns = 8^s, so every index and twiddle stride is a constant shift.
// Twiddles are read from a shared-memory copy of the n-th-root table.
// ---------------------------------------------------------------------------
template <int L>
struct Pow2Plan {
  static constexpr int N = 1 << L;
  static constexpr int TPT = N / kEPT;
  static constexpr int NST = (L + 2) / 3;
  __host__ __device__ static constexpr int radix(int s) {
    return (L - 3 * s >= 3) ? 8 : ((L - 3 * s == 2) ? 4 : 2);
  }
  __host__ __device__ static constexpr int log2radix(int s) {
    return (L - 3 * s >= 3) ? 3 : (L - 3 * s);
  }
};

// Stage twiddle table of a 2^L transform: for every stage S >= 1 the rows
// W^{r k step_S}, r = 1..R_S-1, k = 0..Ns-1, stored [r-1][k] so that lanes
// with consecutive k read consecutive words (a table indexed by r k step
// would put the lanes of a stage-1 butterfly 8 step words apart, all in one
// bank).  At most 2^L entries.
template <int L>
struct StageTw {
  __host__ __device__ static constexpr int off(int S) {
    int o = 0;
    for (int s = 1; s < S; ++s) o += (Pow2Plan<L>::radix(s) - 1) << (3 * s);
    return o;
  }
  static constexpr int size = off(Pow2Plan<L>::NST);
  static_assert(size <= (1 << L), "stage table larger than the transform");
};

// Builds the stage table of a 2^L transform from the global roots of unity of
// order 2^(L+TWS) (caller synchronises before use).
template <typename T, int L, int TWS>
__device__ __forceinline__ void load_stage_twiddles(cplx_t<T> *stg, const cplx_t<T> *__restrict__ tw) {
  using PP = Pow2Plan<L>;
  for (int i = threadIdx.x; i < StageTw<L>::size; i += blockDim.x) {
    int S = 1;
    while (S + 1 < PP::NST && i >= StageTw<L>::off(S + 1)) ++S;
    const int li = i - StageTw<L>::off(S);
    const int lns = 3 * S;
    const int r = (li >> lns) + 1, k = li & ((1 << lns) - 1);
    const int lstep = L - lns - PP::log2radix(S);
    stg[i] = tw[(r * k) << (lstep + TWS)];
  }
}

// exchange barrier: the whole CTA, or only the warp when every transform
// lives inside one warp (its TPT threads are consecutive lanes)
template <bool WSYNC>
__device__ __forceinline__ void xsync() {
  if constexpr (WSYNC) __syncwarp();
  else __syncthreads();
}

// Twiddles of one butterfly, w_r = W^{r k step}, r = 1 .. R-1.  With POW
// (fp64 only) w_1 comes from the stage table and the other powers are formed
// by squaring and multiplying (w2 = w1^2, w3 = w2 w1, w4 = w2^2, w5 = w4 w1,
// w6 = w3^2, w7 = w6 w1: at most three roundings deep, a few ulp), so a
// radix-8 butterfly reads one 16-byte table entry instead of seven.  It trades
// shared-memory bandwidth for fp64 products and about 10-45 registers a
// thread, so only kernels where that measured faster (x forward, fused z) ask
// for it; the others read every power from the table.
template <typename T, int DIR, int R, bool POW>
__device__ __forceinline__ void stage_twiddles(cplx_t<T> (&w)[R], const cplx_t<T> *row1, int NS) {
  if constexpr (sizeof(T) == 8 && POW) {
    w[1] = row1[0];
    if (DIR > 0) w[1].y = -w[1].y;
    if constexpr (R > 2) {
      w[2] = cmul(w[1], w[1]);
      w[3] = cmul(w[2], w[1]);
    }
    if constexpr (R > 4) {
      w[4] = cmul(w[2], w[2]);
      w[5] = cmul(w[4], w[1]);
      w[6] = cmul(w[3], w[3]);
      w[7] = cmul(w[6], w[1]);
    }
  } else {
#pragma unroll
    for (int r = 1; r < R; ++r) {
      w[r] = row1[(r - 1) * NS];
      if (DIR > 0) w[r].y = -w[r].y;
    }
  }
}

// stg: the stage table of the 2^L transform (load_stage_twiddles).
template <typename T, int DIR, int L, int S, bool PAD, int TWS, bool WSYNC = false, bool TWP = false>
__device__ __forceinline__ void ct_stage(cplx_t<T> (&v)[kEPT], int t, const cplx_t<T> *stg,
                                         cplx_t<T> *sbase, int sj) {
  using PP = Pow2Plan<L>;
  constexpr int R = PP::radix(S);
  constexpr int LR = PP::log2radix(S);
  constexpr int B = kEPT / R;
  constexpr int LNS = 3 * S;             // log2 Ns
  constexpr int NS = 1 << LNS;
  constexpr bool LAST = S == PP::NST - 1;
#pragma unroll
  for (int u = 0; u < B; ++u) {
    const int j = t + u * PP::TPT;
    const int k = j & (NS - 1);
    cplx_t<T> a[R];
#pragma unroll
    for (int r = 0; r < R; ++r) a[r] = v[u + r * B];
    if (S > 0) {
      cplx_t<T> w[R];
      stage_twiddles<T, DIR, R, TWP>(w, stg + StageTw<L>::off(S) + k, NS);
#pragma unroll
      for (int r = 1; r < R; ++r) a[r] = cmul(a[r], w[r]);
    }
    dftR<T, DIR, R>(a);
    if (LAST) {
#pragma unroll
      for (int r = 0; r < R; ++r) v[u + r * B] = a[r];
    } else {
      const int idxD = ((j >> LNS) << (LNS + LR)) + k;
#pragma unroll
      for (int r = 0; r < R; ++r) sbase[sidx<PAD>(idxD + r * NS, sj)] = a[r];
    }
  }
  if (!LAST) {
    xsync<WSYNC>();
#pragma unroll
    for (int e = 0; e < kEPT; ++e) v[e] = sbase[sidx<PAD>(t + e * PP::TPT, sj)];
    xsync<WSYNC>();
  }
}

// TWP: twiddle powers formed in registers (stage_twiddles)
template <typename T, int DIR, int L, bool PAD, int TWS = 0, bool WSYNC = false, bool TWP = false, int S = 0>
__device__ __forceinline__ void ct_fft(cplx_t<T> (&v)[kEPT], int t, const cplx_t<T> *stg, cplx_t<T> *sbase,
                                       int sj) {
  if constexpr (S < Pow2Plan<L>::NST) {
    ct_stage<T, DIR, L, S, PAD, TWS, WSYNC, TWP>(v, t, stg, sbase, sj);
    ct_fft<T, DIR, L, PAD, TWS, WSYNC, TWP, S + 1>(v, t, stg, sbase, sj);
  }
}

// copy the n-th roots of unity to shared memory (caller synchronises)
template <typename T>
__device__ __forceinline__ void load_twiddles(cplx_t<T> *stw, const cplx_t<T> *__restrict__ tw, int n) {
  for (int i = threadIdx.x; i < n; i += blockDim.x) stw[i] = tw[i];
}

// padded row length in shared memory
__host__ __device__ constexpr int padded_row(int n) { return n + n / 8; }

// C2C along a strided axis: data viewed as [outer][n][inner]; a CTA owns one
// outer index and `ic` consecutive inner columns; thread (t, c), c fastest.
template <typename T, int DIR, bool PAD>
__global__ void k_cols_reg(cplx_t<T> *__restrict__ data, int64_t inner, int ic, RadixPlan rp,
                           const cplx_t<T> *__restrict__ tw) {
  using C = cplx_t<T>;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  C *sm = reinterpret_cast<C *>(smem_raw);
  const int n = rp.n, TPT = n / kEPT;
  const int c = threadIdx.x % ic, t = threadIdx.x / ic;
  const int64_t nchunks = (inner + ic - 1) / ic;
  const int64_t o = blockIdx.x / nchunks;
  const int64_t i0 = (blockIdx.x - o * nchunks) * ic;
  const bool ok = i0 + c < inner;
  C *base = data + o * (int64_t)n * inner + i0 + c;
  C v[kEPT];
#pragma unroll
  for (int e = 0; e < kEPT; ++e) v[e] = ok ? base[(int64_t)(t + e * TPT) * inner] : cmk<C, T>(T(0), T(0));
  reg_fft<T, DIR, PAD>(v, t, rp, tw, sm + c, ic);
  if (ok) {
#pragma unroll
    for (int e = 0; e < kEPT; ++e) base[(int64_t)(t + e * TPT) * inner] = v[e];
  }
}

// Forward R2C along x: rows of n reals -> n/2+1 complex; thread (t, row), t fastest.
template <typename T>
__global__ void k_rows_r2c_reg(const T *__restrict__ in, cplx_t<T> *__restrict__ out, int64_t nrows,
                               int rpc, RadixPlan rp, const cplx_t<T> *__restrict__ tw) {
  using C = cplx_t<T>;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  C *sm = reinterpret_cast<C *>(smem_raw);
  const int n = rp.n, TPT = n / kEPT, nxh = n / 2 + 1;
  const int t = threadIdx.x % TPT, rr = threadIdx.x / TPT;
  const int64_t row = (int64_t)blockIdx.x * rpc + rr;
  const bool ok = row < nrows;
  C v[kEPT];
#pragma unroll
  for (int e = 0; e < kEPT; ++e) v[e] = cmk<C, T>(ok ? in[row * n + t + e * TPT] : T(0), T(0));
  reg_fft<T, -1, true>(v, t, rp, tw, sm + (size_t)rr * (n + n / 8), 1);
  if (ok) {
#pragma unroll
    for (int e = 0; e < kEPT; ++e) {
      const int idx = t + e * TPT;
      if (idx < nxh) out[row * nxh + idx] = v[e];
    }
  }
}


// Inverse C2R along x of F fields with interleaved real output: a CTA
// transforms all F fields of rpc consecutive mesh rows and writes
// out[(row*n + x)*F + f] (the gather then reads one contiguous run of F*p
// values per stencil row).  Input field f of global row g = frame*nzy + zy
// sits at in[((frame*F + f)*nzy + zy)*nxh].
template <typename T>
__global__ void k_rows_c2r_il(const cplx_t<T> *__restrict__ in, T *__restrict__ out, int F, int64_t nzy,
                              int64_t nrows, int rpc, RadixPlan rp, const cplx_t<T> *__restrict__ tw) {
  using C = cplx_t<T>;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  C *sm = reinterpret_cast<C *>(smem_raw);
  const int n = rp.n, TPT = n / kEPT, nxh = n / 2 + 1;
  const int t = threadIdx.x % TPT, q = threadIdx.x / TPT;
  const int f = q % F, rr = q / F;
  const int64_t row0 = (int64_t)blockIdx.x * rpc;
  const int64_t row = row0 + rr;
  const bool ok = row < nrows;
  const int64_t frame = ok ? row / nzy : 0, zy = ok ? row - frame * nzy : 0;
  const C *src = in + ((frame * F + f) * nzy + zy) * nxh;
  C v[kEPT];
#pragma unroll
  for (int e = 0; e < kEPT; ++e) {
    const int m = t + e * TPT;
    C x = cmk<C, T>(T(0), T(0));
    if (ok) {
      if (m < nxh) {
        x = src[m];
      } else {
        const C h = src[n - m];
        x = cmk<C, T>(h.x, -h.y);
      }
    }
    v[e] = x;
  }
  reg_fft<T, +1, true>(v, t, rp, tw, sm + (size_t)(rr * F + f) * (n + n / 8), 1);
  __syncthreads();
  T *so = reinterpret_cast<T *>(smem_raw);
#pragma unroll
  for (int e = 0; e < kEPT; ++e) so[((size_t)rr * n + t + e * TPT) * F + f] = v[e].x;
  __syncthreads();
  const int64_t nvalid = min((int64_t)rpc, nrows - row0) * n * F;
  T *dst = out + row0 * n * F;
  for (int64_t i = threadIdx.x; i < nvalid; i += blockDim.x) dst[i] = so[i];
}

}  // namespace sogb
