// Host entry of the TMA column FFT passes (fft_tma.cu).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace sogb {

// In-place column FFT of the fp64 spectrum data [outer][n][inner] along n
// (dir -1 forward, +1 inverse, unnormalised) with TMA tile movement, for
// n = 256 or 512.  tw: the n-th roots of unity of the axis.  Returns false,
// without launching anything, when this path does not apply (other n, no
// tensor-map support, alignment); the caller then runs k_cols_pipe.
bool launch_cols_tma(double2 *data, int n, int64_t inner, int64_t outer, int dir, const double2 *tw,
                     unsigned *status, cudaStream_t st);

}  // namespace sogb
