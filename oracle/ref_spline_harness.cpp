// C-ABI harness around the reference's own lmp/sog_spline.h (compiled from the
// reference tree, never copied).  Test infrastructure: pins the oracle's
// B-spline and QuadS weights and the QuadS 1-D influence to the reference.
// sog_spline.h uses std::vector / std::fill without including their headers,
// so they are included first.
#include <algorithm>
#include <vector>
#include "sog_spline.h"

extern "C" {

// lmp/sog_spline.h:19-38 (same recurrence as lmp/sog.cpp:89-110)
void ref_bspline_weights(int n, double t, double *w) {
  std::vector<double> v;
  LAMMPS_NS::fastsog_bspline_weights_1d(n, t, v);
  for (int a = 0; a < n; ++a) w[a] = v[a];
}

// lmp/sog_spline.h:301-304
void ref_quads_weights(int order, double t, double *w) {
  LAMMPS_NS::quads_weights_1d(t, LAMMPS_NS::quads_xi(order), order, w);
}

// lmp/sog_spline.h:327-344
double ref_quads_influence_1d(int m, int n, int order) {
  return LAMMPS_NS::quads_influence_1d(m, n, LAMMPS_NS::quads_xi(order), order);
}

}
