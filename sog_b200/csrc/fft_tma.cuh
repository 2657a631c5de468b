// Blackwell tile movement for the power-of-two column FFTs: TMA
// (cp.async.bulk.tensor) tile loads and stores completed on mbarriers, a
// producer warp that only moves tiles, and transforms that live inside one
// warp (one column per warp, n/32 elements per lane, exchanges through a
// per-warp shared-memory row with warp barriers only).
//
// Every wait on an mbarrier is bounded (one second of %globaltimer); a wait
// that runs out raises a status bit and the kernel drains its own copies and
// returns instead of spinning.  Tensor maps only ever describe this GPU's own
// buffers and no load uses cluster multicast.
#pragma once
#include <cuda.h>

#include "fft_pipe.cuh"

namespace sogb {

// ---- mbarrier and bulk-copy primitives (inline PTX) ----
__device__ __forceinline__ void mbar_init(uint64_t *bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Waits for the phase of `parity` to complete, for at most one second; false
// (and kStatusWaitTimeout raised) when it never does.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, unsigned parity, unsigned *status) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (global_ns() - t0 < 1000000000ull)
    if (mbar_try_wait(bar, parity)) return true;
  raise_status(status, kStatusWaitTimeout);
  return false;
}
// 2-D tiled TMA load into shared memory, completing its bytes on `bar`
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *m, int x, int y, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(m), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *m, int x, int y, const void *src) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(m), "r"(x), "r"(y),
               "r"(smem_u32(src))
               : "memory");
}
// 1-D bulk copies (16-byte aligned addresses, sizes a multiple of 16)
__device__ __forceinline__ void bulk_load_1d(void *dst, const void *src, unsigned bytes, uint64_t *bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void bulk_store_1d(void *dst, const void *src, unsigned bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(smem_u32(src)), "r"(bytes)
               : "memory");
}
// named barrier over `count` threads (a multiple of 32)
__device__ __forceinline__ void named_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// the stores issued so far have finished reading shared memory
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// the stores issued so far are complete
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// generic-proxy shared-memory writes become visible to the bulk-copy (async) proxy
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- warp-resident power-of-two transform ----
// A transform of n = 2^L (L = 8, 9) points lives in one warp: lane t holds
// x[t + 32 e], e < n/32.  Stockham radix-8 (then 4 or 2) stages as in
// ct_stage, with n/32/R butterflies per lane and stage, the exchanges through
// the warp's own padded row (sidx<true>) and __syncwarp only.
template <int L>
struct WarpFft {
  static constexpr int N = 1 << L;
  static constexpr int EPT = N / 32;
  static constexpr int XROW = N + N / 8 + 1;   // padded row + 1: the warps' rows start in different banks
};

template <int DIR, int L, int S>
__device__ __forceinline__ void wf_stage(double2 (&v)[WarpFft<L>::EPT], int t, const double2 *stg, double2 *row) {
  using PP = Pow2Plan<L>;
  constexpr int EPT = WarpFft<L>::EPT;
  constexpr int R = PP::radix(S), LR = PP::log2radix(S), B = EPT / R, LNS = 3 * S, NS = 1 << LNS;
  constexpr bool LAST = S == PP::NST - 1;
#pragma unroll
  for (int u = 0; u < B; ++u) {
    const int j = t + u * 32;
    const int k = j & (NS - 1);
    double2 a[R];
#pragma unroll
    for (int r = 0; r < R; ++r) a[r] = v[u + r * B];
    if (S > 0) {
#pragma unroll
      for (int r = 1; r < R; ++r) {
        double2 w = stg[StageTw<L>::off(S) + (r - 1) * NS + k];
        if (DIR > 0) w.y = -w.y;
        a[r] = cmul(a[r], w);
      }
    }
    dftR<double, DIR, R>(a);
    if (LAST) {
#pragma unroll
      for (int r = 0; r < R; ++r) v[u + r * B] = a[r];
    } else {
      const int idxD = ((j >> LNS) << (LNS + LR)) + k;
#pragma unroll
      for (int r = 0; r < R; ++r) row[sidx<true>(idxD + r * NS, 1)] = a[r];
    }
  }
  if (!LAST) {
    __syncwarp();
#pragma unroll
    for (int e = 0; e < EPT; ++e) v[e] = row[sidx<true>(t + 32 * e, 1)];
    __syncwarp();
  }
}
template <int DIR, int L, int S = 0>
__device__ __forceinline__ void warp_fft(double2 (&v)[WarpFft<L>::EPT], int t, const double2 *stg, double2 *row) {
  if constexpr (S < Pow2Plan<L>::NST) {
    wf_stage<DIR, L, S>(v, t, stg, row);
    warp_fft<DIR, L, S + 1>(v, t, stg, row);
  }
}

// Slot of (row r, column c) in a tile of 8 complex<double> columns as the
// 128-byte swizzled TMA copy lays it out: the 16-byte chunk index of each
// 128-byte row XORed with the row index mod 8 (tile base 1024-byte aligned).
// A warp reading one column then touches eight different chunks per eight
// rows, so the column reads are free of bank conflicts.
__device__ __forceinline__ int tile_slot(int r, int c) { return r * 8 + (c ^ (r & 7)); }

}  // namespace sogb
