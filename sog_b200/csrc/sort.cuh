// Deterministic, stable LSD radix sort of (bin key, atom slot) pairs, and a
// three-phase exclusive scan.  The atoms of a call are cell-sorted with it so
// that the spread accumulates every grid point in a fixed order (bit-for-bit
// reproducible): stability keeps atoms of one bin in slot order.
#pragma once
#include "common.cuh"

namespace sogb {

constexpr int kSortThreads = 256;
constexpr int kSortTile = 4096;  // keys per block per pass
constexpr int kRadixBits = 8;
constexpr int kRadixBuckets = 1 << kRadixBits;

// histogram of one digit over each block's tile -> hist[digit * nblocks + block]
__global__ void k_radix_hist(const uint32_t *__restrict__ keys, int64_t n, int shift,
                             uint32_t *__restrict__ hist, int nblocks) {
  __shared__ uint32_t h[kRadixBuckets];
  for (int i = threadIdx.x; i < kRadixBuckets; i += blockDim.x) h[i] = 0;
  __syncthreads();
  const int64_t base = (int64_t)blockIdx.x * kSortTile;
  const int64_t end = min(n, base + kSortTile);
  for (int64_t i = base + threadIdx.x; i < end; i += blockDim.x)
    atomicAdd(&h[(keys[i] >> shift) & (kRadixBuckets - 1)], 1u);
  __syncthreads();
  for (int i = threadIdx.x; i < kRadixBuckets; i += blockDim.x)
    hist[(int64_t)i * nblocks + blockIdx.x] = h[i];
}

// stable scatter: rank inside the tile = earlier sub-tiles + earlier warps of
// the same sub-tile + earlier lanes with the same digit
__global__ void k_radix_scatter(const uint32_t *__restrict__ kin, const int32_t *__restrict__ vin,
                                uint32_t *__restrict__ kout, int32_t *__restrict__ vout, int64_t n,
                                int shift, const uint32_t *__restrict__ offs, int nblocks) {
  constexpr int W = kSortThreads / 32;
  __shared__ uint32_t wcount[W][kRadixBuckets];
  __shared__ uint32_t run[kRadixBuckets];
  for (int i = threadIdx.x; i < kRadixBuckets; i += blockDim.x)
    run[i] = offs[(int64_t)i * nblocks + blockIdx.x];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t base = (int64_t)blockIdx.x * kSortTile;
  const int64_t end = min(n, base + kSortTile);
  for (int64_t sub = base; sub < end; sub += kSortThreads) {
    for (int i = threadIdx.x; i < W * kRadixBuckets; i += blockDim.x) (&wcount[0][0])[i] = 0;
    __syncthreads();
    const int64_t i = sub + threadIdx.x;
    const bool valid = i < end;
    uint32_t key = 0;
    int32_t val = 0;
    unsigned d = kRadixBuckets;  // sentinel for invalid lanes
    if (valid) {
      key = kin[i];
      val = vin[i];
      d = (key >> shift) & (kRadixBuckets - 1);
    }
    const unsigned peers = __match_any_sync(0xffffffffu, d);
    const unsigned lower = peers & ((1u << lane) - 1u);
    const int lrank = __popc(lower);
    if (valid && lower == 0) wcount[warp][d] = __popc(peers);
    __syncthreads();
    for (int dd = threadIdx.x; dd < kRadixBuckets; dd += blockDim.x) {
      uint32_t s = run[dd];
      for (int w = 0; w < W; ++w) {
        const uint32_t c = wcount[w][dd];
        wcount[w][dd] = s;
        s += c;
      }
      run[dd] = s;
    }
    __syncthreads();
    if (valid) {
      const uint32_t pos = wcount[warp][d] + lrank;
      kout[pos] = key;
      vout[pos] = val;
    }
    __syncthreads();
  }
}

// ---- exclusive scan of uint32 (three phases) ----
constexpr int kScanBlock = 1024;

__device__ __forceinline__ uint32_t block_exclusive_scan(uint32_t v, uint32_t *total) {
  __shared__ uint32_t warp_sums[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    uint32_t s = lane < nw ? warp_sums[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    if (lane < nw) warp_sums[lane] = s;
  }
  __syncthreads();
  const uint32_t before = warp == 0 ? 0 : warp_sums[warp - 1];
  if (total) *total = warp_sums[(blockDim.x >> 5) - 1];
  __syncthreads();
  return before + x - v;
}

__global__ void k_scan_local(const uint32_t *__restrict__ in, uint32_t *__restrict__ out,
                             int64_t n, uint32_t *__restrict__ block_sums) {
  const int64_t i = (int64_t)blockIdx.x * kScanBlock + threadIdx.x;
  const uint32_t v = i < n ? in[i] : 0;
  uint32_t tot;
  const uint32_t ex = block_exclusive_scan(v, &tot);
  if (i < n) out[i] = ex;
  if (threadIdx.x == 0) block_sums[blockIdx.x] = tot;
}

// one block scans the block sums sequentially in chunks
__global__ void k_scan_sums(uint32_t *__restrict__ sums, int64_t nb) {
  __shared__ uint32_t carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int64_t c = 0; c < nb; c += kScanBlock) {
    const int64_t i = c + threadIdx.x;
    const uint32_t v = i < nb ? sums[i] : 0;
    uint32_t tot;
    const uint32_t ex = block_exclusive_scan(v, &tot);
    if (i < nb) sums[i] = ex + carry;
    __syncthreads();
    if (threadIdx.x == 0) carry += tot;
    __syncthreads();
  }
}

__global__ void k_scan_add(uint32_t *__restrict__ out, int64_t n, const uint32_t *__restrict__ sums) {
  const int64_t i = (int64_t)blockIdx.x * kScanBlock + threadIdx.x;
  if (i < n) out[i] += sums[blockIdx.x];
}

// bin_start[b] = first sorted position with key >= b, for b in [0, nbins]
__global__ void k_bin_starts(const uint32_t *__restrict__ skeys, int64_t n, uint32_t nbins,
                             uint32_t *__restrict__ bin_start) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i > n) return;
  const int64_t lo = (i == 0) ? 0 : (int64_t)skeys[i - 1] + 1;
  const int64_t hi = (i == n) ? (int64_t)nbins : (int64_t)skeys[i];
  for (int64_t b = lo; b <= hi; ++b) bin_start[b] = (uint32_t)i;
}

}  // namespace sogb
