// Host entry of the TMA column FFT passes (fft_tma.cu).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "common.cuh"

namespace sogb {

// In-place column FFT of the fp64 spectrum data [outer][n][inner] along n
// (dir -1 forward, +1 inverse, unnormalised) with TMA tile movement, for
// n = 256 or 512.  tw: the n-th roots of unity of the axis.  Returns false,
// without launching anything, when this path does not apply (other n, no
// tensor-map support, alignment); the caller then runs k_cols_pipe.
bool launch_cols_tma(double2 *data, int n, int64_t inner, int64_t outer, int dir, const double2 *tw,
                     unsigned *status, cudaStream_t st);

// Inverse y pass of the field spectra [nf][F][nz][n][inner] with the field
// formation of two-slot frames (k_cols_fields' semantics) through TMA tiles,
// for n = 256 or 512.  False, without launching, when this path does not apply.
bool launch_cols_fields_tma(double2 *data, const FrameGeom *geom, int nf, int F, int nz, int n, int64_t inner,
                            const double2 *tw, int two_slot, int want_pot, unsigned *status, cudaStream_t st);

// Inverse C2R x pass of F fields [nframes][F][nzy][n/2+1] -> interleaved real
// [nframes][nzy][n][F] (k_c2r_pipe's semantics) with bulk-copied rows, for
// n = 512 and F <= 8.  False, without launching, when this path does not apply.
bool launch_c2r_tma(const double2 *in, double *out, int F, int64_t nzy, int64_t nrows, int n, const double2 *tw,
                    unsigned *status, cudaStream_t st);

// Forward R2C x pass of rows of n reals -> n/2+1 complex (k_r2c_pipe's
// semantics) with bulk-copied rows, for n = 512.  False, without launching,
// when this path does not apply.
bool launch_r2c_tma(const double *in, double2 *out, int64_t nrows, int n, const double2 *tw, unsigned *status,
                    cudaStream_t st);

}  // namespace sogb
