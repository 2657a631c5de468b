/*
 * sog_b200.h — C ABI of the B200 (sm_100a) SOG reciprocal-space solver.
 *
 * Plain C: pointers, sizes and integer status codes; no exceptions cross it
 * and no framework types appear in it.  All device arrays are owned by the
 * caller; a plan owns only its scratch (mesh buffers, FFT twiddles, atom-sort
 * buffers).  Work is ordered on the CUDA stream passed in (as void*); no host
 * synchronisation happens inside a forward call except a short wait before a
 * plan reuses its pinned upload buffer.  One plan per stream at a time.
 *
 * Reference interfaces this ABI replaces (paths in the reference project):
 *   - the mesh solve of Gaussian.compute_bundle: src/sog/module/gaussian.py:380-820,
 *     quads_fft.py:209-326 (QuadS) and the B-spline mesh of lmp/sog.cpp:1795-2398;
 *   - its hand-written backward: src/sog/module/cubes2_fft.py:746-869;
 *   - the direct k-sum: src/sog/module/gaussian.py:1180-1337;
 *   - the plugin GPU hooks sog_gpu_create / sog_gpu_setup / sog_gpu_compute
 *     called at lmp/sog.cpp:1049-1053 and lmp/sog.cpp:1804-1836 (their
 *     source, sog_gpu.cu, is not part of the reference).
 */
#ifndef SOG_B200_H
#define SOG_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define SOG_API __attribute__((visibility("default")))
#else
#define SOG_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---- */
#define SOG_OK 0
#define SOG_ERR_INVALID 1     /* bad argument (sizes, orders, null pointers)  */
#define SOG_ERR_CUDA 2        /* a CUDA runtime call failed                   */
#define SOG_ERR_NOMEM 3       /* device or pinned allocation failed           */
#define SOG_ERR_UNSUPPORTED 4 /* valid request this build does not implement  */
#define SOG_ERR_DEVICE 5      /* a kernel raised a status bit (see plan status) */
#define SOG_ERR_COMM 6        /* the caller's exchange callback failed        */

#define SOG_DTYPE_F64 0
#define SOG_DTYPE_F32 1

#define SOG_SPLINE_BSPLINE 0 /* cardinal B-spline, order 4/5/6 (lmp/sog.cpp:89-110) */
#define SOG_SPLINE_QUADS 1   /* separable QuadS, order 4/6 (quads_spline.py)       */
#define SOG_SPLINE_CUBES2 2  /* CubeS2, order 4/6 (cubes2_spline.py, cubes2_fft.py) */

/* Mode -> wave vector.  PHYSICAL: k = 2*pi * cell^-1 * m, the reciprocal
 * vector for cells whose rows are lattice vectors (what the reference's direct
 * path uses, gaussian.py:1040).  REFERENCE: k = 2*pi * m * cell^-1 exactly as
 * written in quads_fft.py:255-257; the two agree whenever cell^-1 is
 * symmetric (orthorhombic cells). */
#define SOG_KCONV_PHYSICAL 0
#define SOG_KCONV_REFERENCE 1

/* plan status bits (sog_plan_status) */
#define SOG_STATUS_NONFINITE 1u /* a position or charge was NaN/Inf           */
#define SOG_STATUS_BAD_CELL 2u  /* a cell had |det| <= eps                    */
#define SOG_STATUS_WAIT_TIMEOUT 4u /* a kernel's wait for its own tile copies ran
                                      out of time (one second); results invalid */

SOG_API const char *sog_strerror(int code);
/* Text of the last failure on this thread (empty string if none). */
SOG_API const char *sog_last_error(void);
/* Library version string. */
SOG_API const char *sog_version(void);
/* Number of kernels this library has launched in the process so far. */
SOG_API unsigned long long sog_launch_count(void);

/* ------------------------------------------------------------------------ */
/* Mesh (particle-mesh) solver                                               */
/* ------------------------------------------------------------------------ */

typedef struct sog_plan sog_plan;

typedef struct sog_plan_desc {
  int dtype;        /* SOG_DTYPE_F64 | SOG_DTYPE_F32                         */
  int spline;       /* SOG_SPLINE_BSPLINE | SOG_SPLINE_QUADS | SOG_SPLINE_CUBES2 */
  int order;        /* 4,5,6 (B-spline) or 4,6 (QuadS, CubeS2)               */
  int nx, ny, nz;   /* mesh; layout [nz][ny][nx], x fastest (quads_fft.py:66) */
  int device;       /* CUDA device ordinal                                   */
  int alias_extent; /* B-spline alias half-width; 0 -> 8 (lmp/sog.cpp:339)   */
  int kconv;        /* SOG_KCONV_*                                           */
} sog_plan_desc;

/* Creates a plan for one mesh shape.  Replaces the reference's per-call
 * grid set-up (quads_fft.py:234-284) and the plugin's ensure_fft_plan /
 * precompute_green_functions (lmp/sog.cpp:892-1096, 1324-1476). */
SOG_API int sog_plan_create(sog_plan **out, const sog_plan_desc *desc);
SOG_API int sog_plan_destroy(sog_plan *plan);
/* Reads and clears the plan's device status bits (synchronises the device). */
SOG_API int sog_plan_status(sog_plan *plan, unsigned *bits);
/* Per-kernel timing: when on, each forward records a CUDA event on the
 * caller's stream after every kernel.  sog_plan_timings waits for the last
 * event, returns up to `cap` (kernel name, ms) pairs of all calls since the
 * previous read (or since timing was switched on) and clears them.  Switching
 * timing on creates a pool of max(2048, on) events, so that calls captured
 * into a CUDA graph (which record one event per kernel per call) create none;
 * a replayed graph re-records its events, so read once per replay. */
SOG_API int sog_plan_set_timing(sog_plan *plan, int on);
SOG_API int sog_plan_timings(sog_plan *plan, const char **names, float *ms, int cap, int *count);

typedef struct sog_mesh_args {
  /* Frames solved by this call (all on this plan's mesh).  Host arrays. */
  int nframes;
  const int64_t *atom_begin; /* [nframes] first atom of each frame            */
  const int64_t *atom_count; /* [nframes] atoms of each frame                 */
  const double *k_sq_max;    /* [nframes] mode cutoff (cubes2_fft.py:102-175) */
  /* Device inputs in the plan's dtype. */
  int nchannels;             /* C: independent charge channels               */
  const void *positions;     /* [N,3] Cartesian                               */
  const void *charges;       /* [N,C]                                         */
  const void *cells;         /* [nframes,3,3], rows = lattice vectors         */
  int n_gauss;               /* M                                             */
  const void *amp;           /* [M] internal amplitudes (amp * bw^2 for raw)  */
  const void *bw2;           /* [M] squared bandwidths                        */
  double norm_factor;        /* 14.3996454784255 by default                   */
  double self_coeff;         /* real-space self term (gaussian.py:210-214)     */
  int remove_self;           /* subtract the mesh self energy                 */
  int k0_correction;         /* add the k=0 term of gaussian.py:769-793       */
  double charge_neutral_lambda; /* > 0 adds lambda*mean(q)^2 (gaussian.py:796) */
  /* Device outputs in the plan's dtype; any may be NULL. */
  void *energy;              /* [nframes]                                     */
  void *forces;              /* [N,3] written for the atoms of these frames   */
  void *potential;           /* [N,C] dE/dq                                   */
  void *grad_amp;            /* [nframes,M] dE/damp                           */
  void *grad_bw2;            /* [nframes,M] dE/dbw2                           */
  void *virial;              /* [nframes,3,3] (cubes2_fft.py:874-921)          */
  /* [N,3] the exact gradient dE/dr of the returned energy: the derivatives of
   * the spline weights on the potential field, which is what torch autograd
   * gives through the reference's QuadS spread (quads_fft.py:34-73); `forces`
   * holds the ik-differentiated explicit forces of quads_fft.py:301-313.
   * B-spline and QuadS meshes; single-device calls only. */
  void *dedr;
} sog_mesh_args;

/* Energy (+ ik forces, dE/dq, dE/d(amp,bw2), virial) of every frame of the
 * call.  Channels are solved independently and summed per frame; the k=0
 * term uses the frame's total charge over channels (gaussian.py:577-654,
 * 769-798).  Replaces compute_quads_fft (quads_fft.py:209-326) and the
 * backward of Cubes2FFTFunction (cubes2_fft.py:746-869). */
SOG_API int sog_mesh_forward(sog_plan *plan, const sog_mesh_args *args, void *stream);

/* ------------------------------------------------------------------------ */
/* One large system over several GPUs: z-slab decomposition                  */
/* ------------------------------------------------------------------------ */
/* Rank r of `size` (one GPU each, every rank with the whole atom set) owns
 * real-space planes [r*nz/size, (r+1)*nz/size) and, after the transpose,
 * half-spectrum rows [r*ny/size, (r+1)*ny/size).  The caller supplies the
 * collective as a callback that must run in stream order on `stream`:
 *   SOG_EXCH_ALLTOALL  send block k (bytes each, at send_off + k*bytes) to
 *                      rank k; receive rank k's block at recv_off + k*bytes;
 *   SOG_EXCH_HALO      send `bytes` at send_off to rank r-1, receive rank
 *                      r+1's `bytes` at recv_off (ranks mod size);
 *   SOG_EXCH_SUM_F64   in-place sum over ranks of bytes/8 doubles at send_off.
 * Offsets are bytes into `workspace`, which has sog_mesh_slab_workspace()
 * bytes at the same layout on every rank.  No counterpart in the reference,
 * which solves the whole mesh on every rank (the plugin's FFT3d spans the
 * full grid on each MPI rank, lmp/sog.cpp:1084-1087). */
#define SOG_EXCH_ALLTOALL 0
#define SOG_EXCH_HALO 1
#define SOG_EXCH_SUM_F64 2
#define SOG_EXCH_ALLGATHER 3   /* `bytes` at send_off from every rank to recv_off + k*bytes */

/* Transports of the transposes and the halo:
 *  SOG_SLAB_EXCHANGE  pack / unpack kernels around the caller's ALLTOALL and
 *                     HALO callbacks (any collective library);
 *  SOG_SLAB_PEER      the column FFT and fused z kernels store straight into
 *                     the other ranks' receive buffers over NVLink (CUDA IPC
 *                     handles swapped once with ALLGATHER); the callbacks then
 *                     only carry ALLGATHER and SUM_F64 (the latter doubles as
 *                     the stream-ordered barrier between the passes).  All
 *                     ranks must be GPUs of one node with peer access; at
 *                     most 8 ranks.  The receive buffers stay exported for
 *                     the plan's life: destroy the plans of a group together. */
#define SOG_SLAB_EXCHANGE 0
#define SOG_SLAB_PEER 1

typedef int (*sog_exchange_fn)(void *ctx, int kind, int64_t send_off, int64_t recv_off, int64_t bytes,
                               void *stream);

typedef struct sog_slab_desc {
  int rank, size;
  int transport;            /* SOG_SLAB_EXCHANGE | SOG_SLAB_PEER              */
  void *workspace;          /* device, sog_mesh_slab_workspace() bytes        */
  size_t workspace_bytes;
  sog_exchange_fn exchange;
  void *ctx;                /* passed back to exchange                       */
} sog_slab_desc;

/* Workspace bytes for a plan split over `size` ranks with `nfield` fields
 * (3 for forces, +1 for dE/dq) and the given transport. */
SOG_API int sog_mesh_slab_workspace(const sog_plan *plan, int nfield, int size, int transport,
                                    size_t *bytes);

/* sog_mesh_forward for one frame split over the ranks of `slab`: energy (the
 * same on every rank), and forces / dE/dq of the atoms whose stencil anchor
 * lies in this rank's planes (the other rows are zeroed; summing the arrays
 * over ranks gives every atom's).  Requires nframes = 1, nz a power of two
 * up to 1024, nz and ny divisible by size, nz/size a multiple of 8 and at
 * least order-1.  Parameter gradients and the virial are not available in
 * this mode (SOG_ERR_UNSUPPORTED). */
SOG_API int sog_mesh_slab_forward(sog_plan *plan, const sog_mesh_args *args, const sog_slab_desc *slab,
                                  void *stream);

/* ------------------------------------------------------------------------ */
/* Direct k-sum                                                              */
/* ------------------------------------------------------------------------ */

typedef struct sog_direct sog_direct;

SOG_API int sog_direct_create(sog_direct **out, int dtype, int device);
SOG_API int sog_direct_destroy(sog_direct *d);
SOG_API int sog_direct_set_timing(sog_direct *d, int on);
SOG_API int sog_direct_timings(sog_direct *d, const char **names, float *ms, int cap, int *count);

typedef struct sog_direct_args {
  int nframes;
  const int64_t *atom_begin; /* host [nframes]                                 */
  const int64_t *atom_count; /* host [nframes]                                 */
  const int32_t *nk;         /* host [nframes,3] integer mode box half-widths  */
  const double *k_sq_max;    /* host [nframes] (2*pi/n_dl)^2                   */
  int nchannels;
  const void *positions, *charges, *cells;
  int n_gauss;
  const void *amp, *bw2;
  double norm_factor, self_coeff;
  int remove_self, k0_correction;
  double charge_neutral_lambda;
  void *energy, *forces, *potential, *grad_amp, *grad_bw2;
  void *virial;              /* [nframes,3,3] reciprocal virial, or NULL        */
} sog_direct_args;

/* E = (1/2V) sum_{k!=0,|k|<=kmax} K(k^2) |S(k)|^2 with explicit derivatives.
 * Replaces _compute_periodic_direct / _compute_bundle_direct_batched
 * (gaussian.py:1180-1337), whose forces the reference takes by autograd. */
SOG_API int sog_direct_forward(sog_direct *d, const sog_direct_args *args, void *stream);

/* Hessian-vector products: the double backward of autograd (a force loss in
 * training differentiates dE/dr again).  For every frame f, with E_f the
 * frame's energy as the forward computes it (all of its terms: the k-space
 * or pair sum, the self term, the k=0 term and the neutrality penalty), and
 * d = (dir_q, dir_r, dir_amp[f], dir_bw2[f]) a direction over the charges,
 * positions and the kernel parameters:
 *   out_q, out_r       = the (charges, positions) rows of H(E_f) d, frame by frame
 *   out_amp[f], out_bw2[f] = the parameter rows of H(E_f) d
 * A NULL direction counts as zero; every output must be given. */
typedef struct sog_hvp_args {
  const void *dir_q;              /* device [N,C], or NULL                       */
  const void *dir_r;              /* device [N,3], or NULL                       */
  const void *dir_amp, *dir_bw2;  /* device [nframes,M], or NULL                 */
  void *out_q;                    /* device [N,C]                                */
  void *out_r;                    /* device [N,3]                                */
  void *out_amp, *out_bw2;        /* device [nframes,M]                          */
} sog_hvp_args;

/* Hessian-vector product of the direct k-sum energy (the second derivatives
 * the reference takes with torch.autograd through _compute_periodic_direct /
 * _compute_bundle_direct_batched, gaussian.py:1180-1337, when forces are
 * built with create_graph=True).  Same inputs as sog_direct_forward (its
 * energy / derivative outputs are ignored). */
SOG_API int sog_direct_hvp(sog_direct *d, const sog_direct_args *args, const sog_hvp_args *h, void *stream);

/* ------------------------------------------------------------------------ */
/* Real-space pair sum (non-periodic frames)                                 */
/* ------------------------------------------------------------------------ */

typedef struct sog_realspace_args {
  int nframes;
  const int64_t *atom_begin; /* host [nframes]                                 */
  const int64_t *atom_count; /* host [nframes]                                 */
  int nchannels;             /* 1..8                                           */
  const void *positions;     /* device [N,3]                                   */
  const void *charges;       /* device [N,C]                                   */
  int n_gauss;
  const void *amp, *bw2;     /* device [M] internal amplitudes, bandwidth^2    */
  double norm_factor;
  int remove_self;           /* 0: add 1/2 sum |q|^2 sum amp                   */
  double charge_neutral_lambda; /* <= 0: no penalty                            */
  void *energy;              /* [nframes]                                      */
  void *forces, *potential;  /* [N,3], [N,C] (dE/dq), or NULL                  */
  void *grad_amp, *grad_bw2; /* [nframes,M], or NULL                           */
  void *virial;              /* [nframes,3,3] written as zeros, or NULL        */
} sog_realspace_args;

/* E_f = norm (1/2 sum_{i != j} (q_i . q_j) sum_m amp_m exp(-r_ij^2 / (2 bw2_m))
 *             + [!remove_self] 1/2 sum_i |q_i|^2 sum_m amp_m) + lambda sum_c mean_c(q)^2
 * over each frame's atoms, with explicit forces, dE/dq and dE/d(amp, bw2).
 * Replaces compute_potential_realspace (gaussian.py:822-845), the path the
 * reference's compute_bundle takes for cell=None and singular cells
 * (gaussian.py:735-746), whose derivatives it takes by autograd.  Runs on a
 * direct-solver context (its scratch and timing); dtype as the context's. */
SOG_API int sog_realspace_forward(sog_direct *d, const sog_realspace_args *args, void *stream);

/* Hessian-vector product of the real-space pair-sum energy (sog_hvp_args as
 * for sog_direct_hvp): the second derivatives the reference takes with
 * torch.autograd through compute_potential_realspace (gaussian.py:822-845). */
SOG_API int sog_realspace_hvp(sog_direct *d, const sog_realspace_args *args, const sog_hvp_args *h,
                              void *stream);

/* Hessian-vector product of the mesh energy (sog_hvp_args as for
 * sog_direct_hvp; the sog_mesh_args outputs are ignored): the second
 * derivatives the reference takes with torch.autograd through its QuadS
 * spread, transforms and gather (compute_quads_fft, quads_fft.py:209-326),
 * for plans of SOG_SPLINE_QUADS and SOG_SPLINE_BSPLINE, whose position
 * gradient is the derivative of the spread weights.  A CubeS2 plan returns
 * SOG_ERR_UNSUPPORTED: the reference's Cubes2FFTFunction backward
 * (cubes2_fft.py:746-869) is the ik force, whose own derivative is not the
 * energy's Hessian. */
SOG_API int sog_mesh_hvp(sog_plan *p, const sog_mesh_args *args, const sog_hvp_args *h, void *stream);

/* ------------------------------------------------------------------------ */
/* Direct k-sum without allocation (no counterpart in the reference)         */
/* ------------------------------------------------------------------------ */

/* Scratch held in one fixed device array per device, and the most frames
 * one call may carry. */
#define SOG_NOALLOC_SCRATCH_BYTES (8u << 20)
#define SOG_NOALLOC_MAX_FRAMES 64

/* Same result as sog_direct_forward (same kernels, same launch shapes, same
 * arguments) on the calling thread's current device, for callers that may
 * not allocate device or pinned host memory inside a force call: an MD
 * engine that hands out device memory only from its own arena and forbids
 * cudaMalloc after setup (cudaMalloc / cudaHostAlloc can wait on queued
 * device work and can fail under memory pressure mid-run), or an integrator
 * that keeps no per-context state.  The call makes no allocation: its
 * scratch is a file-scope __device__ array of SOG_NOALLOC_SCRATCH_BYTES
 * bytes, and the per-frame metadata travels as a kernel parameter.
 *  - status: optional caller-owned device word (NULL: none).  The call sets
 *    it to its status bits (the SOG_STATUS_* bits of sog_plan_status: e.g.
 *    non-finite positions or charges, a singular cell) in stream order; read
 *    it after the stream has passed the call.
 *  - The first call in each CUDA context (per device, and again after
 *    cudaDeviceReset or under another driver-API context) resolves the
 *    array's address there, which may load the module into that context;
 *    make it before any stream capture.
 *  - A call whose scratch would exceed the array (about 48 bytes per mode of
 *    the largest frame's mode box per frame and channel, more with
 *    parameter gradients or the virial), or with more than
 *    SOG_NOALLOC_MAX_FRAMES frames, returns SOG_ERR_INVALID and launches
 *    nothing; sog_last_error() gives the bytes needed.
 *  - Nothing in the scratch has to start at zero: each call writes every
 *    scratch word before reading it.
 *  - All calls on one device share the array: two calls in flight at once
 *    on one device (different streams or host threads) race.  Serialise
 *    them on one stream or with an event. */
SOG_API int sog_direct_forward_noalloc(int dtype, const sog_direct_args *args, unsigned int *status,
                                       void *stream);

#ifdef __cplusplus
}
#endif

#endif /* SOG_B200_H */
