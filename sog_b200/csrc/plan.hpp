// Plan and scratch-buffer management (host side).
#pragma once
#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "common.cuh"
#include "fft.cuh"

namespace sogb {

// A growable device buffer owned by a plan.
struct DevBuf {
  void *p = nullptr;
  size_t bytes = 0;
  int reserve(size_t need);   // SOG_OK or SOG_ERR_NOMEM (contents not kept)
  void release();
  template <typename X> X *as() const { return reinterpret_cast<X *>(p); }
};

// Pinned upload staging buffer; reuse waits on the event of the last copy.
struct PinnedBuf {
  void *p = nullptr;
  size_t bytes = 0;
  cudaEvent_t done = nullptr;
  bool pending = false;
  int reserve(size_t need);
  int wait();
  void release();
};

// Spread tile (threads own (x,y) columns and TZ z-values in registers) and the
// atom-sort bins (cubes of kBin grid cells).
#ifndef SOG_TILE_Z
#define SOG_TILE_Z 8
#endif
constexpr int kTileX = 32, kTileY = 8, kTileZ = SOG_TILE_Z;
constexpr int kBin = 8;

struct AxisTables {
  // Per-axis Green factors (double), one entry per mode index of the axis:
  //   QuadS:    |W_1(m)|^2               (quads_fft.py:150-165)
  //   B-spline: sinc^2p(pi m/N) / S(m)^2  (lmp/sog.cpp:1495-1515)
  // and the B-spline alias sums S(m) for the alias path.
  DevBuf fx, fy, fz, sx, sy, sz;
};

// Optional per-kernel timing: events recorded on the launching stream after
// each kernel of a call (enabled per plan for measurement).
struct Tracer {
  bool on = false;
  std::vector<cudaEvent_t> ev;
  std::vector<const char *> names;
  int used = 0;
  void begin(cudaStream_t st);
  void mark(cudaStream_t st, const char *name);
  void release();
};

void count_launch(int n = 1);

}  // namespace sogb

struct sog_plan {
  sog_plan_desc d{};
  int nxh = 0;
  int64_t ng = 0, nh = 0;  // real / half-spectrum points per frame
  sogb::RadixPlan rpx{}, rpy{}, rpz{};
  sogb::RadixPlan rpxh{};           // nx/2 (even nx: real x rows as half-length transforms)
  sogb::DevBuf twx, twy, twz;   // n-th roots (complex, plan dtype)
  // fp32 plans: the same roots in fp64, for the forward transforms (which
  // run in fp64 for every plan; see mesh_forward_impl)
  sogb::DevBuf twx64, twy64, twz64;
  sogb::AxisTables tab;
  // scratch
  sogb::DevBuf frames_host_dev, geom, status;
  sogb::DevBuf keys0, vals0, keys1, vals1, hist, scan_tmp, bin_start;
  sogb::DevBuf s_atom, s_anchor, s_t, s_q;
  sogb::DevBuf qsum;            // [nf][C][2]  sum q, sum q^2
  sogb::DevBuf rho, spec, fspec, freal;
  sogb::DevBuf partE, partX;    // kspace partial sums
  sogb::DevBuf red;             // reduced sums and per-frame scalars
  sogb::DevBuf redtmp, qpart;   // two-level reduction scratch, charge-sum partials
  sogb::DevBuf btab;            // per-axis kernel factors (orthorhombic frames)
  sogb::DevBuf gtab, gtabF, partD;  // Green tables and self-sum partials of the fused path
  sogb::DevBuf krad;                // radial kernel tables of cubic frames
  // Hessian-vector products: direction spectrum, parameter / self partials,
  // reduced rows, direction sums, per-frame scalars
  sogb::DevBuf hspec, hpart, hred, hdsum, hscal;
  sogb::PinnedBuf up;
  sogb::Tracer tr;
  int nb_x = 0, nb_y = 0, nb_z = 0;  // sort bins per axis
  // z-slab peer transport: receive buffers exported to the other ranks of a
  // group (CUDA IPC) and the peers' buffers mapped here (own rank: local)
  sogb::DevBuf xr_fwd, xr_inv, xr_fe;
  void *peer_fwd[8] = {}, *peer_inv[8] = {}, *peer_fe[8] = {};
  int peer_rank = -1, peer_size = 0;
};

struct sog_direct {
  int dtype = 0, device = 0;
  sogb::DevBuf frames_host_dev, geom, modes, sfac, part, qsum, status, qpart, redtmp;
  // Hessian-vector products: the modes' X sums, per-block partials, reduced
  // sums, direction sums and per-frame scalars
  sogb::DevBuf hx, hpart, hred, hdsum, hscal;
  sogb::PinnedBuf up;
  sogb::Tracer tr;
};

namespace sogb {
void set_error(const std::string &msg);
int fail(int code, const std::string &msg);
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev);
  ~DeviceGuard();
};
void build_radix_plan(int n, RadixPlan *rp);
}  // namespace sogb
