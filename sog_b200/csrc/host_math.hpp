// Host-side spline tables of the product (double precision).
//  - QuadS monomial coefficients: src/sog/module/quads_spline.py:69-158
//  - QuadS 1-D influence |W_1(m)|^2: src/sog/module/quads_fft.py:119-165
//  - B-spline sinc^(2p) alias sums: lmp/sog.cpp:68-76, 1113-1176
#pragma once
#include <cmath>
#include <complex>

namespace sogb {

inline double quads_xi(int order) { return order == 4 ? 1.0 / std::sqrt(3.0) : 0.72879488; }

// coef[k*order + p]: coefficient of t^p of the weight of stencil offset
// 1-order/2+k.  Offsets >= 1 take the published base polynomials; offsets <= 0
// follow from the reflection c_i(t) = c_{1-i}(1-t).
inline void quads_coeffs(int order, double *coef) {
  const double xi = quads_xi(order), x2 = xi * xi, x4 = x2 * x2;
  auto base = [&](int i, double *c) {
    for (int p = 0; p < order; ++p) c[p] = 0.0;
    if (order == 4) {
      if (i == 1) { c[0] = x2 / 2.0; c[1] = -(3.0 * x2 - 2.0) / 2.0; c[2] = 0.5; c[3] = -0.5; }
      else { c[1] = (3.0 * x2 - 1.0) / 6.0; c[3] = 1.0 / 6.0; }
    } else if (i == 1) {
      c[0] = -(3.0 * x4 - 4.0 * x2) / 6.0; c[1] = (5.0 * x4 - 7.0 * x2 + 4.0) / 4.0;
      c[2] = -(3.0 * x2 - 2.0) / 3.0; c[3] = (10.0 * x2 - 7.0) / 12.0;
      c[4] = -1.0 / 6.0; c[5] = 1.0 / 12.0;
    } else if (i == 2) {
      c[0] = (3.0 * x4 - x2) / 24.0; c[1] = -(5.0 * x4 - 7.0 * x2 + 2.0) / 8.0;
      c[2] = (6.0 * x2 - 1.0) / 24.0; c[3] = -(10.0 * x2 - 7.0) / 24.0;
      c[4] = 1.0 / 24.0; c[5] = -1.0 / 24.0;
    } else {
      c[1] = (15.0 * x4 - 15.0 * x2 + 4.0) / 120.0; c[3] = (2.0 * x2 - 1.0) / 24.0;
      c[5] = 1.0 / 120.0;
    }
  };
  const int nu = order / 2;
  for (int k = 0; k < order; ++k) {
    const int off = 1 - nu + k;
    double *c = coef + k * order;
    if (off >= 1) {
      base(off, c);
    } else {
      double b[6];
      base(1 - off, b);
      for (int j = 0; j < order; ++j) {
        double s = 0.0;
        for (int p = j; p < order; ++p) {
          double bin = 1.0;
          for (int i = 1; i <= j; ++i) bin = bin * double(p - j + i) / double(i);
          s += b[p] * bin;
        }
        c[j] = ((j & 1) ? -1.0 : 1.0) * s;
      }
    }
  }
}

inline double quads_influence_1d(int m, int n, int order) {
  using cd = std::complex<double>;
  const double alpha = (2.0 * M_PI / double(n)) * double(m);
  double coef[36];
  quads_coeffs(order, coef);
  cd I[8];
  const cd ia(0.0, alpha);
  if (std::fabs(alpha) < 1e-3) {
    for (int p = 0; p < order; ++p) {
      cd s(1.0 / double(p + 1), 0.0), pw(1.0, 0.0);
      double fact = 1.0;
      for (int k = 1; k < 12; ++k) {
        pw *= ia;
        fact *= double(k);
        s += pw / (fact * double(p + k + 1));
      }
      I[p] = s;
    }
  } else {
    const cd eia = std::exp(ia), inv = 1.0 / ia;
    I[0] = (eia - 1.0) * inv;
    for (int p = 1; p < order; ++p) I[p] = (eia - double(p) * I[p - 1]) * inv;
  }
  const int nu = order / 2;
  cd phi(0.0, 0.0);
  for (int k = 0; k < order; ++k) {
    cd g(0.0, 0.0);
    for (int p = 0; p < order; ++p) g += coef[k * order + p] * I[p];
    phi += std::exp(cd(0.0, alpha * double(1 - nu + k))) * std::conj(g);
  }
  return phi.real() * phi.real() + phi.imag() * phi.imag();
}

inline double sinc(double x) { return std::fabs(x) < 1e-14 ? 1.0 : std::sin(x) / x; }

inline double bspline_sinc2p(int mode, int n, int order, int j) {
  const double arg = M_PI * double(mode) / double(n) + M_PI * double(j);
  return std::pow(sinc(arg), double(2 * order));
}

inline double bspline_sinc_sum(int mode, int n, int order, int extent) {
  double s = 0.0;
  for (int j = -extent; j <= extent; ++j) s += bspline_sinc2p(mode, n, order, j);
  return s;
}

}  // namespace sogb
