// Persistent, software-pipelined versions of the power-of-two FFT passes.
//
// Each CTA loops over tiles (blockIdx.x, +gridDim.x, ...).  While tile i is
// transformed, tile i+1 is already in flight into a second shared-memory
// buffer with cp.async (16-byte LDGSTS, zero-filled past the array end), so
// HBM traffic overlaps the radix-8 arithmetic.  The transform itself is the
// register Stockham of fft_reg.cuh, with its exchanges in a third buffer.
#pragma once
#include <type_traits>
#include "fft_reg.cuh"

namespace sogb {

__device__ __forceinline__ unsigned smem_u32(const void *p) {
  return (unsigned)__cvta_generic_to_shared(p);
}

// 16-byte async copy global -> shared; zero-filled when !valid.
__device__ __forceinline__ void cp_async16(void *dst, const void *src, bool valid) {
  const unsigned d = smem_u32(dst);
  const int sz = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(d), "l"(src), "r"(sz) : "memory");
}
// 8-byte async copy (one complex<float>); zero-filled when !valid.
__device__ __forceinline__ void cp_async8(void *dst, const void *src, bool valid) {
  const unsigned d = smem_u32(dst);
  const int sz = valid ? 8 : 0;
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;\n" ::"r"(d), "l"(src), "r"(sz) : "memory");
}
// one complex element (16 B for double, 8 B for float)
template <typename C>
__device__ __forceinline__ void cp_async_elem(C *dst, const C *src, bool valid) {
  if (sizeof(C) == 16) cp_async16(dst, src, valid);
  else cp_async8(dst, src, valid);
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

// ---------------------------------------------------------------------------
// columns: data [outer][n][inner] complex, tile = (outer o, columns i0..i0+ic)
// ---------------------------------------------------------------------------
// ic is a power of two (the tile widths chosen for power-of-two transforms):
// element q of the tile is row q >> log2(ic), column q & (ic - 1); a thread's
// column is fixed and its rows advance by blockDim.x / ic.
template <typename T>
__device__ __forceinline__ void cols_issue(cplx_t<T> *buf, const cplx_t<T> *data, int64_t inner, int n,
                                           int ic, int64_t nchunks, int64_t tile) {
  using C = cplx_t<T>;
  const int64_t o = tile / nchunks;
  const int64_t i0 = (tile - o * nchunks) * ic;
  const int lic = __ffs(ic) - 1;
  const int col = threadIdx.x & (ic - 1);
  const bool ok = i0 + col < inner;
  const int rstep = blockDim.x >> lic;
  const C *src = data + o * (int64_t)n * inner + i0 + col + (int64_t)(threadIdx.x >> lic) * inner;
  const int64_t sstep = (int64_t)rstep * inner;
  for (int q = threadIdx.x; q < n * ic; q += blockDim.x, src += sstep)
    cp_async_elem(buf + q, ok ? src : data, ok);
}

// Shared memory: 2 input tiles (n*ic), the exchange tile (padded if PAD) and
// the n roots of unity.
template <typename T, int DIR, bool PAD, int L>
__global__ void k_cols_pipe(cplx_t<T> *__restrict__ data, int64_t inner, int ic, int64_t ntiles,
                            const cplx_t<T> *__restrict__ tw) {
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
  int64_t tile = blockIdx.x;
  if (tile < ntiles) cols_issue<T>(buf0, data, inner, n, ic, nchunks, tile);
  cp_async_commit();
  for (int it = 0; tile < ntiles; ++it, tile += gridDim.x) {
    C *cur = (it & 1) ? buf1 : buf0;
    C *nxt = (it & 1) ? buf0 : buf1;
    const int64_t next = tile + gridDim.x;
    if (next < ntiles) cols_issue<T>(nxt, data, inner, n, ic, nchunks, next);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    C v[kEPT];
#pragma unroll
    for (int e = 0; e < kEPT; ++e) v[e] = cur[(t + e * TPT) * ic + c];
    ct_fft<T, DIR, L, PAD>(v, t, stg, xbuf + c, ic);
    const int64_t o = tile / nchunks;
    const int64_t i0 = (tile - o * nchunks) * ic;
    if (i0 + c < inner) {
      C *base = data + o * (int64_t)n * inner + i0 + c;
#pragma unroll
      for (int e = 0; e < kEPT; ++e) base[(int64_t)(t + e * TPT) * inner] = v[e];
    }
    __syncthreads();  // every thread is done with `cur` before it is refilled
  }
  cp_async_wait<0>();
}

// ---------------------------------------------------------------------------
// rows, forward R2C of length n = 2^L as a length n/2 complex FFT
//   z[m] = x[2m] + i x[2m+1],  Z = DFT_{n/2}(z),
//   X[k] = (Z[k] + conj Z[n/2-k]) / 2 - i W_n^k (Z[k] - conj Z[n/2-k]) / 2,
// Z[n/2] = Z[0]; k = 0 .. n/2.  tile = rpc rows; TPT = n/16 threads per row.
// ---------------------------------------------------------------------------
template <typename T, int L>
__global__ void k_r2c_pipe(const T *__restrict__ in, cplx_t<T> *__restrict__ out, int64_t nrows, int rpc,
                           int64_t ntiles, const cplx_t<T> *__restrict__ tw) {
  using C = cplx_t<T>;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  constexpr int n = 1 << L, h = n / 2, TPT = h / kEPT, nxh = h + 1;
  constexpr int hp = padded_row(h);
  T *buf0 = reinterpret_cast<T *>(smem_raw);
  T *buf1 = buf0 + (size_t)rpc * n;
  C *xbuf = reinterpret_cast<C *>(buf1 + (size_t)rpc * n);
  C *stw = xbuf + (size_t)rpc * hp;  // n-th roots of unity (post-processing)
  C *stg = stw + n;                    // stage table of the length n/2 transform
  load_twiddles<T>(stw, tw, n);
  load_stage_twiddles<T, L - 1, 1>(stg, tw);
  const int t = threadIdx.x % TPT, rr = threadIdx.x / TPT;
  constexpr int per = 16 / (int)sizeof(T);
  auto issue = [&](T *buf, int64_t tile) {
    const int64_t row0 = tile * rpc;
    const int64_t valid_rows = min((int64_t)rpc, nrows - row0);
    const int pieces = rpc * n / per;
    const T *src = in + row0 * n;
    for (int q = threadIdx.x; q < pieces; q += blockDim.x) {
      const bool ok = (q * per) / n < valid_rows;
      cp_async16(buf + q * per, ok ? (const void *)(src + q * per) : (const void *)in, ok);
    }
  };
  int64_t tile = blockIdx.x;
  if (tile < ntiles) issue(buf0, tile);
  cp_async_commit();
  C *zrow = xbuf + (size_t)rr * hp;
  for (int it = 0; tile < ntiles; ++it, tile += gridDim.x) {
    T *cur = (it & 1) ? buf1 : buf0;
    T *nxt = (it & 1) ? buf0 : buf1;
    const int64_t next = tile + gridDim.x;
    if (next < ntiles) issue(nxt, next);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    C v[kEPT];
    const T *xr = cur + (size_t)rr * n;
#pragma unroll
    for (int e = 0; e < kEPT; ++e) {
      const int m = t + e * TPT;
      v[e] = cmk<C, T>(xr[2 * m], xr[2 * m + 1]);
    }
    // a row's TPT threads are consecutive lanes of one warp when TPT <= 32
    constexpr bool kWarpRow = TPT <= 32;
    ct_fft<T, -1, L - 1, true, 1, kWarpRow, true>(v, t, stg, zrow, 1);
#pragma unroll
    for (int e = 0; e < kEPT; ++e) zrow[sidx<true>(t + e * TPT, 1)] = v[e];
    xsync<kWarpRow>();
    const int64_t row = tile * rpc + rr;
    if (row < nrows) {
      C *o = out + row * nxh;
#pragma unroll
      for (int e = 0; e < kEPT; ++e) {
        const int k = t + e * TPT;
        const C a = v[e];
        const C b = zrow[sidx<true>((h - k) & (h - 1), 1)];
        const T er = T(0.5) * (a.x + b.x), ei = T(0.5) * (a.y - b.y);   // (Z + conj Z')/2
        const T dr = T(0.5) * (a.x - b.x), di = T(0.5) * (a.y + b.y);   // (Z - conj Z')/2
        const C w = stw[k];                                             // W_n^k
        // -i * w * d
        const T pr = w.x * dr - w.y * di, pi = w.x * di + w.y * dr;
        o[k] = cmk<C, T>(er + pi, ei - pr);
        if (k == 0) o[h] = cmk<C, T>(er - pi, ei + pr);                 // k = n/2: W^{n/2} = -1
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();
}

// ---------------------------------------------------------------------------
// rows, inverse C2R of F fields (interleaved output) as length n/2 complex
// inverse FFTs:  Z[k] = A + i e^{2 pi i k/n} B  with
//   A = X[k] + conj X[n/2-k],  B = X[k] - conj X[n/2-k]   (1 <= k < n/2),
//   Z[0] = (Re X0 + Re Xh) + i (Re X0 - Re Xh),
// then x[2m] = Re z[m], x[2m+1] = Im z[m] for z = IDFT_{n/2}(Z) (unnormalised);
// the imaginary parts of X[0], X[n/2] are ignored as in torch.fft.irfftn.
// ---------------------------------------------------------------------------
template <typename T, int L>
__global__ void k_c2r_pipe(const cplx_t<T> *__restrict__ in, T *__restrict__ out, int F, int64_t nzy,
                           int64_t nrows, int rpc, int64_t ntiles, const cplx_t<T> *__restrict__ tw) {
  using C = cplx_t<T>;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  constexpr int n = 1 << L, h = n / 2, TPT = h / kEPT, nxh = h + 1;
  constexpr int hp = padded_row(h);
  // Two tile buffers: tile i+1 is in flight while tile i is transformed.  A
  // row's slot is wide enough for its exchanges (hp) as well as its input
  // (nxh): once the inputs are in registers the slot serves the transform's
  // exchanges and then the interleaved output, so no third buffer is needed
  // and three CTAs fit on an SM.
  constexpr int rowsz = hp > nxh ? hp : nxh;
  const size_t tsz = (size_t)rpc * F * rowsz;
  C *bufs = reinterpret_cast<C *>(smem_raw);
  C *stw = bufs + 2 * tsz;                 // n-th roots of unity (pre-processing)
  C *stg = stw + n;                        // stage table of the length n/2 transform
  load_twiddles<T>(stw, tw, n);
  load_stage_twiddles<T, L - 1, 1>(stg, tw);
  const int t = threadIdx.x % TPT, q = threadIdx.x / TPT;
  const int f = q % F, rr = q / F;
  auto issue = [&](C *buf, int64_t tile) {
    const int64_t row0 = tile * rpc;
    // one 64-bit division per tile; a thread's (row, field, column) then
    // advances by blockDim.x elements without further divisions
    const int64_t frame0 = row0 / nzy, zy0 = row0 - frame0 * nzy;
    const int total = rpc * F * nxh;
    int hr = threadIdx.x / nxh, col = threadIdx.x - hr * nxh;
    int r2 = hr / F, f2 = hr - r2 * F;
    auto row_src = [&](int rr2, int ff2) -> const C * {
      int64_t frame = frame0, zy = zy0 + rr2;
      while (zy >= nzy) { zy -= nzy; ++frame; }
      return in + ((frame * F + ff2) * nzy + zy) * nxh;
    };
    const C *rsrc = row_src(r2, f2);
    for (int qq = threadIdx.x; qq < total; qq += blockDim.x) {
      const bool ok = row0 + r2 < nrows;
      cp_async_elem(buf + (size_t)(r2 * F + f2) * rowsz + col, ok ? rsrc + col : in, ok);
      col += blockDim.x;
      if (col >= nxh) {
        do {
          col -= nxh;
          if (++f2 == F) { f2 = 0; ++r2; }
        } while (col >= nxh);
        rsrc = row_src(r2, f2);
      }
    }
  };
  int64_t tile = blockIdx.x;
  if (tile < ntiles) issue(bufs, tile);
  cp_async_commit();
  for (int it = 0; tile < ntiles; ++it, tile += gridDim.x) {
    C *cur = bufs + (size_t)(it & 1) * tsz;
    const int64_t next = tile + gridDim.x;
    if (next < ntiles) issue(bufs + (size_t)((it + 1) & 1) * tsz, next);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    C *X = cur + (size_t)(rr * F + f) * rowsz;
    C v[kEPT];
#pragma unroll
    for (int e = 0; e < kEPT; ++e) {
      const int k = t + e * TPT;
      if (k == 0) {
        const T x0 = X[0].x, xh = X[h].x;
        v[e] = cmk<C, T>(x0 + xh, x0 - xh);
      } else {
        const C a = X[k], b = X[h - k];
        const T Ar = a.x + b.x, Ai = a.y - b.y;      // X[k] + conj X[h-k]
        const T Br = a.x - b.x, Bi = a.y + b.y;      // X[k] - conj X[h-k]
        const C w = stw[k];                          // e^{-2 pi i k/n}; use its conjugate
        const T cr = w.x * Br + w.y * Bi, ci = w.x * Bi - w.y * Br;   // conj(w) * B
        v[e] = cmk<C, T>(Ar - ci, Ai + cr);          // A + i conj(w) B
      }
    }
    __syncthreads();   // the tile's inputs are in registers: its slots become exchange space
    ct_fft<T, +1, L - 1, true, 1, (TPT <= 32)>(v, t, stg, X, 1);
    // interleave the F fields of the tile's rows in the same slots (free once
    // every thread is past its transform), then store the tile's contiguous
    // output with vector stores
    __syncthreads();
    T *so = reinterpret_cast<T *>(cur);
#pragma unroll
    for (int e = 0; e < kEPT; ++e) {
      const int m = t + e * TPT;
      so[((size_t)rr * n + 2 * m) * F + f] = v[e].x;
      so[((size_t)rr * n + 2 * m + 1) * F + f] = v[e].y;
    }
    __syncthreads();
    {
      using V2 = typename std::conditional<sizeof(T) == 8, double2, float2>::type;
      const int64_t row0 = tile * rpc;
      const int nv = (int)min((int64_t)rpc, nrows - row0);
      const int cnt = nv * n * F / 2;
      const V2 *src = reinterpret_cast<const V2 *>(so);
      V2 *dst = reinterpret_cast<V2 *>(out + row0 * n * F);
      for (int i = threadIdx.x; i < cnt; i += blockDim.x) dst[i] = src[i];
    }
    __syncthreads();
  }
  cp_async_wait<0>();
}

}  // namespace sogb

namespace sogb {

// ---------------------------------------------------------------------------
// Address maps for the column passes of the slab decomposition.  Element x of
// row `r` of outer slab `o` lives at
//   tab[b] + b*bstride + (o / osplit)*ohi + (o % osplit)*olo + (r - b*rb)*rstride
//          + (x / cw)*cstride + x % cw,                             b = r / rb,
// which covers the plain layout [outer][n][inner] (rb = n, olo = n*inner,
// rstride = inner, cw = cstride = 1), the transposed blocks stored straight
// into the peers' receive buffers (one base pointer per destination rank) in
// the column-chunked layout, and those blocks read back in place.  rb, osplit
// and cw are powers of two (slab sizes divide power-of-two axes): the
// divisions are shifts (rb_sh, os_sh, cw_sh, set by with_shifts), since the
// column passes evaluate this map for every element they move.
// ---------------------------------------------------------------------------
constexpr int kMaxSlabRanks = 8;

template <typename C>
struct RowMap {
  C *tab[kMaxSlabRanks];
  int rb, osplit, cw;
  int64_t bstride, ohi, olo, rstride, cstride;
  int rb_sh, os_sh, cw_sh;
  __device__ __forceinline__ C *at(int64_t o, int r, int64_t x) const {
    const int b = r >> rb_sh;
    const int64_t oh = o >> os_sh, xc = x >> cw_sh;
    return tab[b] + b * bstride + oh * ohi + (o - (oh << os_sh)) * olo + (int64_t)(r - (b << rb_sh)) * rstride +
           xc * cstride + (x - (xc << cw_sh));
  }
};

inline int log2_exact(int v) {
  int s = 0;
  while ((1 << s) < v) ++s;
  return (1 << s) == v ? s : -1;
}

// the map with its shifts set; false if rb, osplit or cw is not a power of two
template <typename C>
inline bool with_shifts(RowMap<C> &m) {
  m.rb_sh = log2_exact(m.rb);
  m.os_sh = log2_exact(m.osplit);
  m.cw_sh = log2_exact(m.cw);
  return m.rb_sh >= 0 && m.os_sh >= 0 && m.cw_sh >= 0;
}

template <typename C>
inline RowMap<C> plain_map(C *base, int n, int64_t inner) {
  RowMap<C> m{};
  m.tab[0] = base;
  m.rb = n;
  m.osplit = 1 << 30;
  m.cw = 1;
  m.bstride = 0;
  m.ohi = 0;
  m.olo = (int64_t)n * inner;
  m.rstride = inner;
  m.cstride = 1;
  with_shifts(m);
  return m;
}

// Column FFT (length 2^L) of the tiles [o][*][i0 .. i0+ic) from `in` to
// `out`, both addressed through row maps.  Same pipeline as k_cols_pipe;
// stores may go to another GPU's memory over NVLink (made visible to the
// peers by a system-scope fence before the kernel ends).
template <typename T, int DIR, bool PAD, int L>
__global__ void k_cols_map(RowMap<cplx_t<T>> in, RowMap<cplx_t<T>> out, int64_t inner, int ic, int64_t ntiles,
                           const cplx_t<T> *__restrict__ tw) {
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
  auto issue = [&](C *buf, int64_t tile) {
    const int64_t o = tile / nchunks;
    const int64_t i0 = (tile - o * nchunks) * ic;
    const int total = n * ic, ic_sh = __ffs(ic) - 1;   // ic: a power of two
    for (int q = threadIdx.x; q < total; q += blockDim.x) {
      const int r = q >> ic_sh, col = q - (r << ic_sh);
      const bool ok = i0 + col < inner;
      const C *src = in.at(o, r, i0 + col);
      cp_async_elem(buf + q, ok ? src : in.tab[0], ok);
    }
  };
  int64_t tile = blockIdx.x;
  if (tile < ntiles) issue(buf0, tile);
  cp_async_commit();
  for (int it = 0; tile < ntiles; ++it, tile += gridDim.x) {
    C *cur = (it & 1) ? buf1 : buf0;
    C *nxt = (it & 1) ? buf0 : buf1;
    const int64_t next = tile + gridDim.x;
    if (next < ntiles) issue(nxt, next);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    C v[kEPT];
#pragma unroll
    for (int e = 0; e < kEPT; ++e) v[e] = cur[(t + e * TPT) * ic + c];
    ct_fft<T, DIR, L, PAD>(v, t, stg, xbuf + c, ic);
    const int64_t o = tile / nchunks;
    const int64_t i0 = (tile - o * nchunks) * ic;
    if (i0 + c < inner) {
#pragma unroll
      for (int e = 0; e < kEPT; ++e) *out.at(o, t + e * TPT, i0 + c) = v[e];
    }
    __syncthreads();
  }
  cp_async_wait<0>();
  __threadfence_system();
}

}  // namespace sogb
