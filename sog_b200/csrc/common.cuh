// Shared device helpers for the SOG B200 library (sm_100a).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/sog_b200.h"

namespace sogb {

constexpr double kPi = 3.14159265358979323846;
constexpr int kMaxOrder = 6;      // largest spline order (p^3 = 216 nodes)
constexpr int kMaxGauss = 64;     // Gaussian terms per kernel (M)

template <typename T> struct Cplx;
template <> struct Cplx<double> { using type = double2; };
template <> struct Cplx<float> { using type = float2; };
template <typename T> using cplx_t = typename Cplx<T>::type;

template <typename C> __device__ __forceinline__ C cmul(C a, C b) {
  C r;
  r.x = a.x * b.x - a.y * b.y;
  r.y = a.x * b.y + a.y * b.x;
  return r;
}
template <typename C> __device__ __forceinline__ C cadd(C a, C b) {
  C r; r.x = a.x + b.x; r.y = a.y + b.y; return r;
}
template <typename C> __device__ __forceinline__ C csub(C a, C b) {
  C r; r.x = a.x - b.x; r.y = a.y - b.y; return r;
}
template <typename C, typename T> __device__ __forceinline__ C cmk(T x, T y) {
  C r; r.x = x; r.y = y; return r;
}

// Per-frame geometry, written on the device from the caller's cells.
struct FrameGeom {
  double cell[9];     // rows = lattice vectors
  double cinv[9];     // inverse cell
  double kmat[9];     // k = kmat * m  (row a holds d k_a / d m_b), includes 2*pi
  double vol;         // |det cell|
  double kmin2;       // min |b_i|^2 over reciprocal vectors (k=0 correction)
  double k_sq_max;    // mode cutoff
  double abound[3];   // |m_a| bound of aliases inside the k_max sphere
  double scale;       // N_g / V (spread charge scale, quads_fft.py:287)
  int64_t atom_begin; // first atom of the frame in the caller's arrays
  int64_t slot_base;  // first sorted slot of the frame
  int32_t natoms;
  int32_t pad;        // 1: B-spline aliases may fall inside the k_max sphere
  int32_t ortho;      // 1: kmat diagonal (k_a depends on m_a only)
  int32_t pad2;
  double sig2[3];     // CubeS2: (xi |a_alpha| / n_alpha)^2 of the Green factor, else 0
};

// Per-frame host-side description uploaded with each call.
struct FrameHost {
  int64_t atom_begin;
  int64_t natoms;
  int64_t slot_base;
  double k_sq_max;
};

// Status bits a kernel may raise (read back by sog_plan_status).
enum : unsigned {
  kStatusNonFinite = 1u << 0,
  kStatusBadCell = 1u << 1,
  kStatusWaitTimeout = 1u << 2,
};

__device__ __forceinline__ void raise_status(unsigned *status, unsigned bit) {
  if (status) atomicOr(status, bit);
}

// Mode index convention of torch.fft (Nyquist at +n/2): quads_fft.py:246-252.
__device__ __forceinline__ int signed_mode(int i, int n) { return i <= n / 2 ? i : i - n; }

}  // namespace sogb

#define SOG_CUDA_TRY(expr)                                          \
  do {                                                              \
    cudaError_t _e = (expr);                                        \
    if (_e != cudaSuccess) { sogb_set_cuda_error(_e); return SOG_ERR_CUDA; } \
  } while (0)

void sogb_set_cuda_error(cudaError_t e);
