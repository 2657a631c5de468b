// Persistent, software-pipelined versions of the power-of-two FFT passes.
//
// Each CTA loops over tiles (blockIdx.x, +gridDim.x, ...).  While tile i is
// transformed, tile i+1 is already in flight into a second shared-memory
// buffer with cp.async (16-byte LDGSTS, zero-filled past the array end), so
// HBM traffic overlaps the radix-8 arithmetic.  The transform itself is the
// register Stockham of fft_reg.cuh, with its exchanges in a third buffer.
#pragma once
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
template <typename T>
__device__ __forceinline__ void cols_issue(cplx_t<T> *buf, const cplx_t<T> *data, int64_t inner, int n,
                                           int ic, int64_t nchunks, int64_t tile) {
  using C = cplx_t<T>;
  const int64_t o = tile / nchunks;
  const int64_t i0 = (tile - o * nchunks) * ic;
  const C *base = data + o * (int64_t)n * inner + i0;
  const int total = n * ic;
  for (int q = threadIdx.x; q < total; q += blockDim.x) {
    const int row = q / ic, col = q - row * ic;
    const bool ok = i0 + col < inner;
    cp_async_elem(buf + q, ok ? base + (int64_t)row * inner + col : data, ok);
  }
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
  C *stw = xbuf + (size_t)(PAD ? padded_row(n) : n) * ic;
  load_twiddles<T>(stw, tw, n);
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
    ct_fft<T, DIR, L, PAD>(v, t, stw, xbuf + c, ic);
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
// rows, forward R2C: tile = rpc rows of n reals
// ---------------------------------------------------------------------------
template <typename T, int L>
__global__ void k_r2c_pipe(const T *__restrict__ in, cplx_t<T> *__restrict__ out, int64_t nrows, int rpc,
                           int64_t ntiles, const cplx_t<T> *__restrict__ tw) {
  using C = cplx_t<T>;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  constexpr int n = 1 << L, TPT = n / kEPT, nxh = n / 2 + 1;
  T *buf0 = reinterpret_cast<T *>(smem_raw);
  T *buf1 = buf0 + (size_t)rpc * n;
  C *xbuf = reinterpret_cast<C *>(buf1 + (size_t)rpc * n);
  C *stw = xbuf + (size_t)rpc * padded_row(n);
  load_twiddles<T>(stw, tw, n);
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
  for (int it = 0; tile < ntiles; ++it, tile += gridDim.x) {
    T *cur = (it & 1) ? buf1 : buf0;
    T *nxt = (it & 1) ? buf0 : buf1;
    const int64_t next = tile + gridDim.x;
    if (next < ntiles) issue(nxt, next);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    C v[kEPT];
#pragma unroll
    for (int e = 0; e < kEPT; ++e) v[e] = cmk<C, T>(cur[rr * n + t + e * TPT], T(0));
    ct_fft<T, -1, L, true>(v, t, stw, xbuf + (size_t)rr * padded_row(n), 1);
    const int64_t row = tile * rpc + rr;
    if (row < nrows) {
#pragma unroll
      for (int e = 0; e < kEPT; ++e) {
        const int idx = t + e * TPT;
        if (idx < nxh) out[row * nxh + idx] = v[e];
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();
}

// ---------------------------------------------------------------------------
// rows, inverse C2R of F fields with interleaved output (see k_rows_c2r_il)
// ---------------------------------------------------------------------------
// Shared memory: 2 input tiles (rpc*F half rows), the exchange / output
// staging area and the n roots of unity.
template <typename T, int L>
__global__ void k_c2r_pipe(const cplx_t<T> *__restrict__ in, T *__restrict__ out, int F, int64_t nzy,
                           int64_t nrows, int rpc, int64_t ntiles, const cplx_t<T> *__restrict__ tw) {
  using C = cplx_t<T>;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  constexpr int n = 1 << L, TPT = n / kEPT, nxh = n / 2 + 1;
  const int hrow = nxh;
  C *buf0 = reinterpret_cast<C *>(smem_raw);
  C *buf1 = buf0 + (size_t)rpc * F * hrow;
  C *xbuf = buf1 + (size_t)rpc * F * hrow;  // exchanges, then the interleaved output staging
  const size_t xsz = max((size_t)rpc * F * padded_row(n) * sizeof(C), (size_t)rpc * n * F * sizeof(T));
  C *stw = reinterpret_cast<C *>(reinterpret_cast<unsigned char *>(xbuf) + ((xsz + 15) & ~(size_t)15));
  load_twiddles<T>(stw, tw, n);
  const int t = threadIdx.x % TPT, q = threadIdx.x / TPT;
  const int f = q % F, rr = q / F;
  auto issue = [&](C *buf, int64_t tile) {
    const int64_t row0 = tile * rpc;
    const int total = rpc * F * nxh;
    for (int qq = threadIdx.x; qq < total; qq += blockDim.x) {
      const int hr = qq / nxh, col = qq - hr * nxh;
      const int r2 = hr / F, f2 = hr - r2 * F;
      const int64_t row = row0 + r2;
      const bool ok = row < nrows;
      const int64_t frame = ok ? row / nzy : 0, zy = ok ? row - frame * nzy : 0;
      const C *src = in + ((frame * F + f2) * nzy + zy) * nxh + col;
      cp_async_elem(buf + (size_t)hr * hrow + col, ok ? src : in, ok);
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
    const C *h = cur + (size_t)(rr * F + f) * hrow;
    C v[kEPT];
#pragma unroll
    for (int e = 0; e < kEPT; ++e) {
      const int m = t + e * TPT;
      if (m < nxh) {
        v[e] = h[m];
      } else {
        const C x = h[n - m];
        v[e] = cmk<C, T>(x.x, -x.y);
      }
    }
    ct_fft<T, +1, L, true>(v, t, stw, xbuf + (size_t)(rr * F + f) * padded_row(n), 1);
    __syncthreads();
    T *so = reinterpret_cast<T *>(xbuf);
#pragma unroll
    for (int e = 0; e < kEPT; ++e) so[((size_t)rr * n + t + e * TPT) * F + f] = v[e].x;
    __syncthreads();
    const int64_t row0 = tile * rpc;
    const int64_t nvalid = min((int64_t)rpc, nrows - row0) * n * F;
    T *dst = out + row0 * n * F;
    for (int64_t i = threadIdx.x; i < nvalid; i += blockDim.x) dst[i] = so[i];
    __syncthreads();
  }
  cp_async_wait<0>();
}

}  // namespace sogb
