/*
 * sog_oracle.c — CPU restatement of SOG's Gaussian reciprocal-space solver.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * library in sog_b200/csrc: the tests, __graft_entry__.smoke() and the
 * cpu_baseline / reference arm of bench.py load it.  The product path never
 * calls it and there is no CPU fallback built on it.
 *
 * Parity anchors (paths relative to the reference project root):
 *   - QuadS weights        src/sog/module/quads_spline.py:69-158
 *   - QuadS influence      src/sog/module/quads_fft.py:119-197
 *   - QuadS pipeline       src/sog/module/quads_fft.py:209-326
 *   - B-spline weights     lmp/sog.cpp:89-110 (same recurrence as
 *                          lmp/sog_spline.h:19-38, which oracle/_ref compiles)
 *   - B-spline Green       lmp/sog.cpp:1113-1176 (sinc tables) and
 *                          lmp/sog.cpp:1479-1578 (principal / alias sums)
 *   - B-spline stencil     lmp/sog.cpp:1977-2018 (offsets ix0-(p-1)/2+a)
 *   - ik forces, potential lmp/sog.cpp:2111-2127, quads_fft.py:301-313
 *   - backward (dq, amp, bw2) src/sog/module/cubes2_fft.py:746-869
 *   - virial               src/sog/module/cubes2_fft.py:874-921
 *   - direct k-sum         src/sog/module/gaussian.py:1281-1337
 *   - real-space pair sum  src/sog/module/gaussian.py:822-845 (frames with
 *                          cell=None or a singular cell, gaussian.py:735-746)
 *   - mode convention      quads_fft.py:246-258 (Nyquist at +N/2)
 *   - irfftn semantics     torch.fft.irfftn: C2C over z,y then C2R along x
 *                          using Re() of the mx=0 / mx=nx/2 columns
 *
 * Parity status: QuadS, CubeS2, direct and real-space paths are pinned against fixtures made by
 * importing the reference (tests/golden/make_golden.py); the B-spline weights
 * are pinned against the reference's own compiled sog_spline.h
 * (oracle/_ref).  The B-spline Green function has no executable reference
 * (lmp/sog.cpp needs LAMMPS); it is restated here from the source.
 *
 * Everything is double precision.  Plain C99 + OpenMP.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_PI 3.14159265358979323846

/* ------------------------------------------------------------------------ */
/* spline weights                                                            */
/* ------------------------------------------------------------------------ */

/* Cardinal B-spline weights of order n at fractional offset t (Cox-de Boor).
 * w[a] is the weight of grid node ix0-(n-1)/2+a.  lmp/sog.cpp:89-110. */
void orc_bspline_weights(int n, double t, double *w) {
  double prev[8];
  for (int a = 0; a < n; ++a) w[a] = 0.0;
  w[0] = 1.0 - t;
  w[1] = t;
  for (int k = 3; k <= n; ++k) {
    const double inv = 1.0 / (double)(k - 1);
    for (int a = 0; a < n; ++a) prev[a] = w[a];
    w[k - 1] = t * prev[k - 2] * inv;
    for (int j = 1; j <= k - 2; ++j)
      w[k - 1 - j] = ((t + (double)j) * prev[k - 2 - j] +
                      ((double)(k - j) - t) * prev[k - 1 - j]) * inv;
    w[0] = (1.0 - t) * prev[0] * inv;
  }
}

/* d w[a] / dt of the order-n B-spline weights: the derivative of the
 * cardinal B-spline, M_n'(x) = M_{n-1}(x) - M_{n-1}(x - 1), i.e.
 * w_n'[a] = w_{n-1}[a-1] - w_{n-1}[a] at the same offset t (the exact
 * derivative of the recurrence above). */
void orc_bspline_dweights(int n, double t, double *dw) {
  double w1[8];
  orc_bspline_weights(n - 1, t, w1);
  for (int a = 0; a < n; ++a) dw[a] = (a >= 1 ? w1[a - 1] : 0.0) - (a < n - 1 ? w1[a] : 0.0);
}

/* QuadS xi for order 4/6: quads_spline.py:12-13 (Table I). */
double orc_quads_xi(int order) {
  return order == 4 ? 1.0 / sqrt(3.0) : 0.72879488;
}

/* Ascending monomial coefficients of the base polynomials c_1..c_nu
 * (quads_spline.py:95-125), then the per-offset table with the reflection
 * c_i(t) = c_{1-i}(1-t) (quads_spline.py:128-163).  coef[k*order + p] is the
 * coefficient of t^p for offset index k (offset = 1-nu+k). */
static void quads_base(int i, double xi, int order, double *c) {
  const double x2 = xi * xi, x4 = x2 * x2;
  for (int p = 0; p < order; ++p) c[p] = 0.0;
  if (order == 4) {
    if (i == 1) {
      c[0] = x2 / 2.0; c[1] = -(3.0 * x2 - 2.0) / 2.0; c[2] = 0.5; c[3] = -0.5;
    } else {
      c[1] = (3.0 * x2 - 1.0) / 6.0; c[3] = 1.0 / 6.0;
    }
  } else {
    if (i == 1) {
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
  }
}

static double binom_d(int n, int k) {
  double r = 1.0;
  for (int i = 1; i <= k; ++i) r = r * (double)(n - k + i) / (double)i;
  return r;
}

void orc_quads_coeffs(int order, double *coef) {
  const double xi = orc_quads_xi(order);
  const int nu = order / 2;
  for (int k = 0; k < order; ++k) {
    const int off = 1 - nu + k;
    double *c = coef + k * order;
    if (off >= 1) {
      quads_base(off, xi, order, c);
    } else {
      double b[6];
      quads_base(1 - off, xi, order, b);
      for (int j = 0; j < order; ++j) {
        double s = 0.0;
        for (int p = j; p < order; ++p) s += b[p] * binom_d(p, j);
        c[j] = ((j & 1) ? -1.0 : 1.0) * s;
      }
    }
  }
}

void orc_quads_weights(int order, double t, double *w) {
  double coef[36];
  orc_quads_coeffs(order, coef);
  for (int k = 0; k < order; ++k) {
    double v = 0.0, tp = 1.0;
    for (int p = 0; p < order; ++p) { v += coef[k * order + p] * tp; tp *= t; }
    w[k] = v;
  }
}

/* d w[k] / dt of the QuadS weights (the derivative of the polynomials). */
void orc_quads_dweights(int order, double t, double *dw) {
  double coef[36];
  orc_quads_coeffs(order, coef);
  for (int k = 0; k < order; ++k) {
    double v = 0.0, tp = 1.0;
    for (int p = 1; p < order; ++p) { v += (double)p * coef[k * order + p] * tp; tp *= t; }
    dw[k] = v;
  }
}

/* |W_1(m)|^2 of the separable QuadS window: quads_fft.py:119-165. */
double orc_quads_influence_1d(int m, int n, int order) {
  const double alpha = (2.0 * ORC_PI / (double)n) * (double)m;
  double coef[36];
  orc_quads_coeffs(order, coef);
  const int deg = order;
  /* I_p(alpha) = int_0^1 t^p e^{i alpha t} dt */
  double Ire[8], Iim[8];
  if (fabs(alpha) < 1e-3) {
    for (int p = 0; p < deg; ++p) {
      double sre = 1.0 / (double)(p + 1), sim = 0.0;
      double pre = 1.0, pim = 0.0, fact = 1.0;
      for (int k = 1; k < 12; ++k) {
        /* pw *= i*alpha */
        const double nre = -pim * alpha, nim = pre * alpha;
        pre = nre; pim = nim;
        fact *= (double)k;
        sre += pre / (fact * (double)(p + k + 1));
        sim += pim / (fact * (double)(p + k + 1));
      }
      Ire[p] = sre; Iim[p] = sim;
    }
  } else {
    const double ere = cos(alpha), eim = sin(alpha);
    /* 1/(i a) = -i/a */
    const double ire = 0.0, iim = -1.0 / alpha;
    double are = ere - 1.0, aim = eim;
    Ire[0] = are * ire - aim * iim; Iim[0] = are * iim + aim * ire;
    for (int p = 1; p < deg; ++p) {
      are = ere - (double)p * Ire[p - 1];
      aim = eim - (double)p * Iim[p - 1];
      Ire[p] = are * ire - aim * iim; Iim[p] = are * iim + aim * ire;
    }
  }
  const int nu = order / 2;
  double phre = 0.0, phim = 0.0;
  for (int k = 0; k < order; ++k) {
    const int off = 1 - nu + k;
    double gre = 0.0, gim = 0.0;
    for (int p = 0; p < deg; ++p) {
      gre += coef[k * order + p] * Ire[p];
      gim += coef[k * order + p] * Iim[p];
    }
    /* e^{i alpha off} * conj(g) */
    const double cr = cos(alpha * (double)off), ci = sin(alpha * (double)off);
    phre += cr * gre + ci * gim;
    phim += ci * gre - cr * gim;
  }
  return phre * phre + phim * phim;
}

/* sinc(x)^(2p) table value and alias sum (lmp/sog.cpp:68-76, 1113-1176). */
/* ------------------------------------------------------------------------ */
/* CubeS2 splines (cubes2_spline.py:16-406; Predescu et al., JCP 153, 224117) */
/* ------------------------------------------------------------------------ */

/* xi of order 4 / 6: cubes2_spline.py:18-19. */
double orc_cubes2_xi(int order) {
  return order == 6 ? 0.6503998764035732 : 1.0 / sqrt(3.0);
}

/* One assignment node: offset d from the floor grid index, symmetry class,
 * special (or, for class 3, normal) axis and the sign bits of the special
 * coordinates (cubes2_spline.py:44-56, 170-228). */
typedef struct { int d[3], cls, sp, neg; } c2node;

static int c2_is01(int c) { return c == 0 || c == 1; }

/* The node table: order 4, classes {0,1}^3 and one axis at -1 or 2
 * (cubes2_spline.py:60-97); order 6, the points of [-2,3]^3 within squared
 * distance 4 of the unit cube, classified by their coordinate pattern
 * (cubes2_spline.py:170-228).  Returns the number of nodes. */
int orc_cubes2_nodes(int order, int *d_out, int *cls_out) {
  int n = 0;
  const int lo = order == 6 ? -2 : -1, hi = order == 6 ? 3 : 2;
  for (int dx = lo; dx <= hi; ++dx)
    for (int dy = lo; dy <= hi; ++dy)
      for (int dz = lo; dz <= hi; ++dz) {
        const int c[3] = {dx, dy, dz};
        double dist = 0.0;
        int nsp = 0;
        for (int a = 0; a < 3; ++a) {
          if (c[a] < 0) dist += (double)c[a] * c[a];
          if (c[a] > 1) dist += (double)(c[a] - 1) * (c[a] - 1);
          if (!c2_is01(c[a])) ++nsp;
        }
        const int keep = order == 6 ? dist <= 4.0 + 1e-10
                                    : (nsp == 0 || (nsp == 1 && dist <= 1.0 + 1e-10));
        if (!keep) continue;
        if (d_out) { d_out[3 * n] = dx; d_out[3 * n + 1] = dy; d_out[3 * n + 2] = dz; }
        if (cls_out) cls_out[n] = nsp;
        ++n;
      }
  return n;
}

static void c2_classify(int order, const int *c, c2node *nd) {
  nd->d[0] = c[0]; nd->d[1] = c[1]; nd->d[2] = c[2];
  int sp[3], nsp = 0;
  for (int a = 0; a < 3; ++a) if (!c2_is01(c[a])) sp[nsp++] = a;
  nd->sp = -1; nd->neg = 0;
  if (nsp == 0) { nd->cls = 0; return; }
  if (nsp == 1) {
    const int a = sp[0];
    nd->sp = a;
    if (c[a] == -1 || c[a] == 2) { nd->cls = 1; nd->neg = c[a] == -1; }
    else { nd->cls = 2; nd->neg = c[a] == -2; }
    (void)order;
    return;
  }
  if (nsp == 2) {   /* class 3: sp holds the normal axis, bits the sorted special axes */
    nd->cls = 3;
    for (int a = 0; a < 3; ++a) if (a != sp[0] && a != sp[1]) nd->sp = a;
    for (int i = 0; i < 2; ++i) if (c[sp[i]] == -1) nd->neg |= 1 << i;
    return;
  }
  nd->cls = 4;
  for (int a = 0; a < 3; ++a) if (c[a] == -1) nd->neg |= 1 << a;
}

/* Eq. 15 / 16 of the paper (cubes2_spline.py:99-110) */
static double c2_L4(double t, double xi) {
  const double x2 = xi * xi;
  return -0.5 * t * t * t + 0.5 * t * t - (9.0 * x2 - 2.0) / 6.0 * t + 0.5 * x2;
}
static double c2_R(double t, double xi) {
  return t * t * t / 6.0 + (3.0 * xi * xi - 1.0) / 6.0 * t;
}
/* order-6 pieces (cubes2_spline.py:126-166) */
static double c2_L111(double t, double xi) {
  const double x2 = xi * xi, x4 = x2 * x2;
  const double t2 = t * t, t3 = t2 * t;
  return t3 * t2 / 12.0 - t2 * t2 / 6.0 + (10.0 * x2 - 1.0) / 12.0 * t3 - (6.0 * x2 - 1.0) / 6.0 * t2 +
         (5.0 * x4 - x2) / 4.0 * t - (3.0 * x4 - x2) / 6.0;
}
static double c2_L311(double t, double xi) {
  const double x2 = xi * xi, x4 = x2 * x2;
  const double t3 = t * t * t;
  return t3 * t * t / 120.0 + (2.0 * x2 - 1.0) / 24.0 * t3 + (15.0 * x4 - 15.0 * x2 + 4.0) / 120.0 * t;
}
static double c2_L211(double t, double xi) { return -0.25 * c2_L111(t, xi) - 2.5 * c2_L311(t, xi); }
static double c2_S6(double t, double xi) {
  const double x2 = xi * xi;
  return -0.5 * t * t * t + 0.5 * t * t - (3.0 * x2 - 2.0) / 2.0 * t + 0.5 * x2;
}

/* eta of a coordinate at a node offset in {0,1}: t at offset 1, 1 - t at 0 */
static double c2_eta01(double t, int d) { return d == 1 ? t : 1.0 - t; }

/* Weight of one node at fractional offsets t[3] in [0,1)
 * (cubes2_weight_4 / cubes2_weight_6, cubes2_spline.py:231-380). */
static double c2_weight(int order, const double *t, const c2node *nd, double xi) {
  const int *d = nd->d;
  if (order == 4) {
    if (nd->cls == 0) {
      const double ex = c2_eta01(t[0], d[0]), ey = c2_eta01(t[1], d[1]), ez = c2_eta01(t[2], d[2]);
      return c2_L4(ex, xi) * ey * ez + c2_L4(ey, xi) * ez * ex + c2_L4(ez, xi) * ex * ey;
    }
    const int s = nd->sp;
    const double es = nd->neg ? 1.0 - t[s] : t[s];
    double prod = 1.0;
    for (int a = 0; a < 3; ++a) if (a != s) prod *= c2_eta01(t[a], d[a]);
    return c2_R(es, xi) * prod;
  }
  switch (nd->cls) {
    case 0: {
      const double ex = c2_eta01(t[0], d[0]), ey = c2_eta01(t[1], d[1]), ez = c2_eta01(t[2], d[2]);
      return c2_L111(ex, xi) * ey * ez + c2_L111(ey, xi) * ez * ex + c2_L111(ez, xi) * ex * ey +
             c2_S6(ex, xi) * c2_S6(ey, xi) * c2_S6(ez, xi);
    }
    case 1: case 2: {
      const int s = nd->sp;
      const double es = nd->neg ? 1.0 - t[s] : t[s];
      double en[2];
      int k = 0;
      for (int a = 0; a < 3; ++a) if (a != s) en[k++] = c2_eta01(t[a], d[a]);
      if (nd->cls == 2) return c2_L311(es, xi) * en[0] * en[1];
      return c2_L211(es, xi) * en[0] * en[1] + c2_R(es, xi) * c2_S6(en[0], xi) * c2_S6(en[1], xi);
    }
    case 3: {
      const int nrm = nd->sp;
      int sa[2], k = 0;
      for (int a = 0; a < 3; ++a) if (a != nrm) sa[k++] = a;
      const double en = c2_eta01(t[nrm], d[nrm]);
      const double e1 = (nd->neg & 1) ? 1.0 - t[sa[0]] : t[sa[0]];
      const double e2 = (nd->neg & 2) ? 1.0 - t[sa[1]] : t[sa[1]];
      return c2_S6(en, xi) * c2_R(e1, xi) * c2_R(e2, xi);
    }
    default: {
      const double ex = (nd->neg & 1) ? 1.0 - t[0] : t[0];
      const double ey = (nd->neg & 2) ? 1.0 - t[1] : t[1];
      const double ez = (nd->neg & 4) ? 1.0 - t[2] : t[2];
      return c2_R(ex, xi) * c2_R(ey, xi) * c2_R(ez, xi);
    }
  }
}

/* Weights of all nodes at fractional offsets t (w[node] in table order). */
int orc_cubes2_weights(int order, const double *t, double *w) {
  int d[3 * 216], cls[216];
  const int n = orc_cubes2_nodes(order, d, cls);
  const double xi = orc_cubes2_xi(order);
  for (int i = 0; i < n; ++i) {
    c2node nd;
    c2_classify(order, d + 3 * i, &nd);
    w[i] = c2_weight(order, t, &nd, xi);
  }
  return n;
}

static double orc_sinc(double x) {
  if (fabs(x) < 1e-14) return 1.0;
  return sin(x) / x;
}

double orc_bspline_sinc2p(int mode, int n, int order, int j) {
  const double arg = ORC_PI * (double)mode / (double)n + ORC_PI * (double)j;
  return pow(orc_sinc(arg), (double)(2 * order));
}

double orc_bspline_sinc_sum(int mode, int n, int order, int alias_extent) {
  double s = 0.0;
  for (int j = -alias_extent; j <= alias_extent; ++j)
    s += orc_bspline_sinc2p(mode, n, order, j);
  return s;
}

/* ------------------------------------------------------------------------ */
/* mixed-radix complex FFT (any 2,3,5-smooth length; generic small primes)   */
/* ------------------------------------------------------------------------ */

typedef struct { double re, im; } cplx;

static int smallest_factor(int n) {
  for (int p = 2; p * p <= n; ++p)
    if (n % p == 0) return p;
  return n;
}

/* out[k] = sum_j in[j*stride] * exp(sign*2*pi*i*j*k/n); recursive DIT.
 * W[j*ws] = exp(sign*2*pi*i*j/n) for j in [0, n) (a root table of a multiple
 * of n read with stride ws). */
static void fft_rec(const cplx *in, int stride, cplx *out, int n, const cplx *W, int ws,
                    cplx *scratch) {
  if (n == 1) { out[0] = in[0]; return; }
  const int p = smallest_factor(n);
  const int m = n / p;
  for (int r = 0; r < p; ++r)
    fft_rec(in + r * stride, stride * p, scratch + r * m, m, W, ws * p, out);
  for (int k = 0; k < m; ++k) {
    for (int q = 0; q < p; ++q) {
      const int kk = k + q * m;
      double sre = 0.0, sim = 0.0;
      for (int r = 0; r < p; ++r) {
        const long e = ((long)r * (long)kk) % n;
        const cplx w = W[e * ws];
        const cplx y = scratch[r * m + k];
        sre += y.re * w.re - y.im * w.im;
        sim += y.re * w.im + y.im * w.re;
      }
      out[kk].re = sre; out[kk].im = sim;
    }
  }
}

static cplx *root_table(int n, int sign) {
  cplx *W = malloc(sizeof(cplx) * n);
  for (int j = 0; j < n; ++j) {
    const long double a = (long double)sign * 2.0L * 3.141592653589793238462643383279502884L *
                          (long double)j / (long double)n;
    W[j].re = (double)cosl(a);
    W[j].im = (double)sinl(a);
  }
  return W;
}

/* In-place 1-D transform of a strided line. */
static void fft_line(cplx *base, long stride, int n, const cplx *W, cplx *w1, cplx *w2, cplx *w3) {
  for (int j = 0; j < n; ++j) w1[j] = base[(long)j * stride];
  fft_rec(w1, 1, w2, n, W, 1, w3);
  for (int j = 0; j < n; ++j) base[(long)j * stride] = w2[j];
}

/* Forward R2C over a [nz][ny][nx] real grid into [nz][ny][nx/2+1]. */
static void orc_rfft3(const double *rho, cplx *out, int nx, int ny, int nz) {
  const int nxh = nx / 2 + 1;
  const int nmax = nx > ny ? (nx > nz ? nx : nz) : (ny > nz ? ny : nz);
  cplx *Wx = root_table(nx, -1), *Wy = root_table(ny, -1), *Wz = root_table(nz, -1);
#pragma omp parallel
  {
    cplx *w1 = malloc(sizeof(cplx) * nmax), *w2 = malloc(sizeof(cplx) * nmax),
         *w3 = malloc(sizeof(cplx) * nmax), *row = malloc(sizeof(cplx) * nmax);
#pragma omp for schedule(static)
    for (long zy = 0; zy < (long)nz * ny; ++zy) {
      for (int x = 0; x < nx; ++x) { row[x].re = rho[zy * nx + x]; row[x].im = 0.0; }
      fft_rec(row, 1, w2, nx, Wx, 1, w3);
      for (int x = 0; x < nxh; ++x) out[zy * nxh + x] = w2[x];
    }
#pragma omp for schedule(static)
    for (long zx = 0; zx < (long)nz * nxh; ++zx) {
      const long z = zx / nxh, x = zx % nxh;
      fft_line(out + z * ny * nxh + x, nxh, ny, Wy, w1, w2, w3);
    }
#pragma omp for schedule(static)
    for (long yx = 0; yx < (long)ny * nxh; ++yx)
      fft_line(out + yx, (long)ny * nxh, nz, Wz, w1, w2, w3);
    free(w1); free(w2); free(w3); free(row);
  }
  free(Wx); free(Wy); free(Wz);
}

/* Unnormalised inverse matching torch.fft.irfftn(X, s=(nz,ny,nx)) * N:
 * C2C inverse over z and y, then C2R along x using Re() of the self-conjugate
 * columns (the imaginary part of mx=0 and mx=nx/2 is ignored). */
static void orc_irfft3(cplx *spec, double *out, int nx, int ny, int nz) {
  const int nxh = nx / 2 + 1;
  const int nmax = nx > ny ? (nx > nz ? nx : nz) : (ny > nz ? ny : nz);
  cplx *Wx = root_table(nx, +1), *Wy = root_table(ny, +1), *Wz = root_table(nz, +1);
#pragma omp parallel
  {
    cplx *w1 = malloc(sizeof(cplx) * nmax), *w2 = malloc(sizeof(cplx) * nmax),
         *w3 = malloc(sizeof(cplx) * nmax), *row = malloc(sizeof(cplx) * nmax);
#pragma omp for schedule(static)
    for (long yx = 0; yx < (long)ny * nxh; ++yx)
      fft_line(spec + yx, (long)ny * nxh, nz, Wz, w1, w2, w3);
#pragma omp for schedule(static)
    for (long zx = 0; zx < (long)nz * nxh; ++zx) {
      const long z = zx / nxh, x = zx % nxh;
      fft_line(spec + z * ny * nxh + x, nxh, ny, Wy, w1, w2, w3);
    }
#pragma omp for schedule(static)
    for (long zy = 0; zy < (long)nz * ny; ++zy) {
      const cplx *h = spec + zy * nxh;
      for (int x = 0; x < nxh; ++x) row[x] = h[x];
      for (int m = 1; m < (nx + 1) / 2; ++m) { row[nx - m].re = h[m].re; row[nx - m].im = -h[m].im; }
      fft_rec(row, 1, w2, nx, Wx, 1, w3);
      for (int x = 0; x < nx; ++x) out[zy * nx + x] = w2[x].re;
    }
    free(w1); free(w2); free(w3); free(row);
  }
  free(Wx); free(Wy); free(Wz);
}

/* exported for the FFT self-test against numpy */
void orc_fft_c2c(const double *in_ri, double *out_ri, int n, int sign) {
  cplx *a = malloc(sizeof(cplx) * n), *b = malloc(sizeof(cplx) * n),
       *c = malloc(sizeof(cplx) * n);
  memcpy(a, in_ri, sizeof(cplx) * n);
  cplx *W = root_table(n, sign);
  fft_rec(a, 1, b, n, W, 1, c);
  free(W);
  memcpy(out_ri, b, sizeof(cplx) * n);
  free(a); free(b); free(c);
}
void orc_rfftn(const double *rho, double *out_ri, int nx, int ny, int nz) {
  orc_rfft3(rho, (cplx *)out_ri, nx, ny, nz);
}
void orc_irfftn_unnorm(double *spec_ri, double *out, int nx, int ny, int nz) {
  orc_irfft3((cplx *)spec_ri, out, nx, ny, nz);
}

/* ------------------------------------------------------------------------ */
/* mesh solve                                                                */
/* ------------------------------------------------------------------------ */

enum { ORC_BSPLINE = 0, ORC_QUADS = 1, ORC_CUBES2 = 2 };

typedef struct {
  int spline, order, nx, ny, nz, alias_extent;
  int kconv;           /* 0: k = 2pi cell^-1 m (physical), 1: k = 2pi m cell^-1 */
  int natoms;
  const double *r;     /* [N,3] */
  const double *q;     /* [N]   */
  double cell[9];      /* rows = lattice vectors */
  int M;
  const double *amp, *bw2;
  double k_sq_max, norm_factor, self_coeff;
  int remove_self, want_force, want_pot, want_param_grad, want_virial;
  int want_dedr;       /* exact dE/dr of the mesh energy (spline-weight derivatives) */
} orc_mesh_in;

typedef struct {
  double energy;     /* mesh energy incl. self terms, times norm (no k=0) */
  double diag_sum;   /* sum_half w*Gself / (2V) */
  double *forces;    /* [N,3] or NULL */
  double *potential; /* [N]  dE/dq incl. self terms, or NULL */
  double *grad_amp;  /* [M] or NULL */
  double *grad_bw2;  /* [M] or NULL */
  double virial[9];
  double *dedr;      /* [N,3] exact dE/dr, or NULL (B-spline and QuadS) */
} orc_mesh_out;

static void inv3(const double *c, double *ci, double *det_out) {
  const double a = c[0], b = c[1], cc = c[2], d = c[3], e = c[4], f = c[5],
               g = c[6], h = c[7], i = c[8];
  const double A = e * i - f * h, B = -(d * i - f * g), C = d * h - e * g;
  const double det = a * A + b * B + cc * C;
  const double id = 1.0 / det;
  ci[0] = A * id; ci[1] = -(b * i - cc * h) * id; ci[2] = (b * f - cc * e) * id;
  ci[3] = B * id; ci[4] = (a * i - cc * g) * id;  ci[5] = -(a * f - cc * d) * id;
  ci[6] = C * id; ci[7] = -(a * h - b * g) * id;  ci[8] = (a * e - b * d) * id;
  *det_out = det;
}

static void atom_stencil(int spline, int order, const double *ci, const double *r,
                         int nx, int ny, int nz, int *i0, double *wx, double *wy,
                         double *wz) {
  const int n3[3] = {nx, ny, nz};
  double *ws[3] = {wx, wy, wz};
  for (int a = 0; a < 3; ++a) {
    double f = r[0] * ci[0 * 3 + a] + r[1] * ci[1 * 3 + a] + r[2] * ci[2 * 3 + a];
    f = f - floor(f);                 /* torch.remainder(., 1.0) */
    const double fx = f * (double)n3[a];
    const double fl = floor(fx);
    const double t = fx - fl;
    int ib = (int)fl;
    /* first stencil node = base + (1 - nu) for QuadS / base - (p-1)/2 */
    const int first = (spline == ORC_QUADS) ? (1 - order / 2) : -((order - 1) / 2);
    ib += first;
    ib %= n3[a]; if (ib < 0) ib += n3[a];
    i0[a] = ib;
    if (spline == ORC_QUADS) orc_quads_weights(order, t, ws[a]);
    else orc_bspline_weights(order, t, ws[a]);
  }
}

/* CubeS2 stencil of one atom: floor grid index per axis (no offset) and the
 * node weights (cubes2_fft.py:408-470). */
static int c2_stencil(int order, const double *ci, const double *r, int nx, int ny, int nz,
                      int *i0, double *w) {
  const int n3[3] = {nx, ny, nz};
  double t[3];
  for (int a = 0; a < 3; ++a) {
    double f = r[0] * ci[0 * 3 + a] + r[1] * ci[1 * 3 + a] + r[2] * ci[2 * 3 + a];
    f = f - floor(f);
    const double fx = f * (double)n3[a];
    const double fl = floor(fx);
    t[a] = fx - fl;
    i0[a] = (int)fl % n3[a];
  }
  return orc_cubes2_weights(order, t, w);
}

/* Green-function factors at one half-spectrum mode.
 * kv: k vector of the principal mode; returns kfac (bare kernel K(k^2)),
 * gE (energy green), gF (force green), gS (self green), gV (virial green),
 * kfacv (bare K_v), and per-Gaussian e_m*D factors for parameter gradients
 * in em_d[M] (energy) and em_s[M] (self).  Returns 0 when the mode is masked.*/
typedef struct {
  int spline, order, alias_extent, nx, ny, nz, M, kconv;
  const double *amp, *bw2;
  double k_sq_max;
  double ci[9];
  double bound[3];    /* |a_alpha| * kmax / 2pi: alias pruning */
  double *dx, *dy, *dz;   /* separable deconvolution per axis */
  double *sx, *sy, *sz;   /* B-spline alias sums per axis */
  double sig2[3];         /* CubeS2: (xi |a_alpha| / n_alpha)^2 */
} green_ctx;

/* Mode m -> Cartesian k.  kconv 0: k = 2pi cell^-1 m, the reciprocal vector
 * for rows-are-lattice-vectors cells (as the direct path, gaussian.py:1040);
 * kconv 1: k = 2pi m cell^-1, the form written in quads_fft.py:255-257, which
 * equals the former only when cell^-1 is symmetric. */
static void kvec(const green_ctx *g, double mx, double my, double mz, double *k) {
  const double tp = 2.0 * ORC_PI;
  for (int a = 0; a < 3; ++a) {
    if (g->kconv)
      k[a] = tp * (mx * g->ci[0 * 3 + a] + my * g->ci[1 * 3 + a] + mz * g->ci[2 * 3 + a]);
    else
      k[a] = tp * (mx * g->ci[a * 3 + 0] + my * g->ci[a * 3 + 1] + mz * g->ci[a * 3 + 2]);
  }
}

static int green_at(const green_ctx *g, int mx, int my, int mz, int iy, int iz,
                    double *kout, double *kfac, double *gE, double *gF,
                    double *gS, double *gV, double *kfacv, double *emD,
                    double *emS, double *emDb, double *emSb) {
  double k[3];
  kvec(g, mx, my, mz, k);
  const double ksq = k[0] * k[0] + k[1] * k[1] + k[2] * k[2];
  kout[0] = k[0]; kout[1] = k[1]; kout[2] = k[2];
  if ((mx == 0 && my == 0 && mz == 0) || ksq > g->k_sq_max) return 0;
  double K = 0.0, Kv = 0.0;
  for (int m = 0; m < g->M; ++m) {
    const double e = exp(-0.5 * g->bw2[m] * ksq);
    K += g->amp[m] * e;
    Kv += g->amp[m] * g->bw2[m] * e;
  }
  *kfac = K; *kfacv = Kv;
  if (g->spline == ORC_CUBES2) {
    /* variance subtraction, G = K exp(sum_a sigma_a^2 k_a^2) over the
     * Cartesian components (cubes2_fft.py:1039-1049) */
    const double D = exp(g->sig2[0] * k[0] * k[0] + g->sig2[1] * k[1] * k[1] + g->sig2[2] * k[2] * k[2]);
    *gE = K * D; *gF = K * D; *gS = K; *gV = Kv * D;
    if (emD) for (int m = 0; m < g->M; ++m) {
      const double e = exp(-0.5 * g->bw2[m] * ksq);
      emD[m] = e * D; emS[m] = e;
      emDb[m] = -0.5 * ksq * emD[m]; emSb[m] = -0.5 * ksq * e;
    }
    return 1;
  }
  if (g->spline == ORC_QUADS) {
    double infl = g->dx[mx] * g->dy[iy] * g->dz[iz];
    if (infl < 1e-20) infl = 1e-20;           /* quads_fft.py:194 clamp */
    const double D = 1.0 / infl;
    *gE = K * D; *gF = K * D; *gS = K; *gV = Kv * D;
    if (emD) for (int m = 0; m < g->M; ++m) {
      const double e = exp(-0.5 * g->bw2[m] * ksq);
      emD[m] = e * D; emS[m] = e;
      emDb[m] = -0.5 * ksq * emD[m]; emSb[m] = -0.5 * ksq * e;
    }
    return 1;
  }
  /* B-spline: sum over aliases q_j = k + 2pi (N*j) . cell_inv inside the
   * k_max sphere (lmp/sog.cpp:1479-1578; the fast path is the j=0 term). */
  const double denom_lin = g->sx[mx] * g->sy[iy] * g->sz[iz];
  const double denom = denom_lin * denom_lin;
  if (!(denom > 1e-20) || !isfinite(denom)) return 0;
  const int E = g->alias_extent;
  const int m3[3] = {mx, my, mz};
  const int n3[3] = {g->nx, g->ny, g->nz};
  int jlo[3], jhi[3];
  for (int a = 0; a < 3; ++a) {
    int lo = (int)ceil((-g->bound[a] - (double)m3[a]) / (double)n3[a]);
    int hi = (int)floor((g->bound[a] - (double)m3[a]) / (double)n3[a]);
    if (lo < -E) lo = -E;
    if (hi > E) hi = E;
    if (lo > 0) lo = 0;   /* principal is always inside */
    if (hi < 0) hi = 0;
    jlo[a] = lo; jhi[a] = hi;
  }
  double sum0 = 0.0, sum1 = 0.0, sumv = 0.0;
  if (emD) for (int m = 0; m < g->M; ++m) { emD[m] = 0.0; emS[m] = 0.0; emDb[m] = 0.0; emSb[m] = 0.0; }
  const double w0 = orc_bspline_sinc2p(mx, g->nx, g->order, 0) *
                    orc_bspline_sinc2p(my, g->ny, g->order, 0) *
                    orc_bspline_sinc2p(mz, g->nz, g->order, 0);
  for (int jx = jlo[0]; jx <= jhi[0]; ++jx)
    for (int jy = jlo[1]; jy <= jhi[1]; ++jy)
      for (int jz = jlo[2]; jz <= jhi[2]; ++jz) {
        double q[3];
        kvec(g, mx + g->nx * jx, my + g->ny * jy, mz + g->nz * jz, q);
        const double qsq = q[0] * q[0] + q[1] * q[1] + q[2] * q[2];
        if (!(qsq > 0.0 && qsq <= g->k_sq_max)) continue;
        double Kq = 0.0, Kvq = 0.0;
        for (int m = 0; m < g->M; ++m) {
          const double e = exp(-0.5 * g->bw2[m] * qsq);
          Kq += g->amp[m] * e;
          Kvq += g->amp[m] * g->bw2[m] * e;
        }
        const double wp = orc_bspline_sinc2p(mx, g->nx, g->order, jx) *
                          orc_bspline_sinc2p(my, g->ny, g->order, jy) *
                          orc_bspline_sinc2p(mz, g->nz, g->order, jz);
        sum0 += Kq * wp;
        sum1 += (k[0] * q[0] + k[1] * q[1] + k[2] * q[2]) * Kq * wp;
        sumv += Kvq * wp;
        if (emD) for (int m = 0; m < g->M; ++m) {
          /* an alias term's bw2 derivative carries its own -|q|^2 / 2 */
          const double e = exp(-0.5 * g->bw2[m] * qsq);
          const double eD = e * wp / denom, eS = (w0 > 1e-20) ? e * wp / w0 : 0.0;
          emD[m] += eD;
          emS[m] += eS;
          emDb[m] += -0.5 * qsq * eD;
          emSb[m] += -0.5 * qsq * eS;
        }
      }
  *gE = sum0 / denom;
  *gF = sum1 / (ksq * denom);
  *gS = (w0 > 1e-20) ? sum0 / w0 : 0.0;
  *gV = sumv / denom;
  return 1;
}

static void setup_green(green_ctx *g, const orc_mesh_in *in, const double *ci) {
  g->spline = in->spline; g->order = in->order; g->alias_extent = in->alias_extent;
  g->nx = in->nx; g->ny = in->ny; g->nz = in->nz; g->M = in->M;
  g->amp = in->amp; g->bw2 = in->bw2; g->k_sq_max = in->k_sq_max;
  g->kconv = in->kconv;
  memcpy(g->ci, ci, sizeof(double) * 9);
  {
    const int n3[3] = {in->nx, in->ny, in->nz};
    const double xi = orc_cubes2_xi(in->order);
    for (int a = 0; a < 3; ++a) {
      const double la = sqrt(in->cell[3 * a] * in->cell[3 * a] + in->cell[3 * a + 1] * in->cell[3 * a + 1] +
                             in->cell[3 * a + 2] * in->cell[3 * a + 2]);
      const double s = xi * la / n3[a];
      g->sig2[a] = s * s;
    }
  }
  const double kmax = sqrt(in->k_sq_max);
  /* |m_a| <= |v_a| kmax / 2pi with v_a the lattice row (kconv 0) or the
   * column of the cell (kconv 1): bounds the aliases inside the sphere. */
  for (int a = 0; a < 3; ++a) {
    double s = 0.0;
    for (int b = 0; b < 3; ++b) {
      const double v = in->kconv ? in->cell[3 * b + a] : in->cell[3 * a + b];
      s += v * v;
    }
    g->bound[a] = sqrt(s) * kmax / (2.0 * ORC_PI) + 1e-9;
  }
  const int nxh = in->nx / 2 + 1;
  g->dx = malloc(sizeof(double) * nxh);
  g->dy = malloc(sizeof(double) * in->ny);
  g->dz = malloc(sizeof(double) * in->nz);
  g->sx = malloc(sizeof(double) * nxh);
  g->sy = malloc(sizeof(double) * in->ny);
  g->sz = malloc(sizeof(double) * in->nz);
  for (int ix = 0; ix < nxh; ++ix) {
    g->dx[ix] = (in->spline == ORC_QUADS) ? orc_quads_influence_1d(ix, in->nx, in->order) : 0.0;
    g->sx[ix] = orc_bspline_sinc_sum(ix, in->nx, in->order, in->alias_extent);
  }
  for (int iy = 0; iy < in->ny; ++iy) {
    const int my = iy <= in->ny / 2 ? iy : iy - in->ny;
    g->dy[iy] = (in->spline == ORC_QUADS) ? orc_quads_influence_1d(my, in->ny, in->order) : 0.0;
    g->sy[iy] = orc_bspline_sinc_sum(my, in->ny, in->order, in->alias_extent);
  }
  for (int iz = 0; iz < in->nz; ++iz) {
    const int mz = iz <= in->nz / 2 ? iz : iz - in->nz;
    g->dz[iz] = (in->spline == ORC_QUADS) ? orc_quads_influence_1d(mz, in->nz, in->order) : 0.0;
    g->sz[iz] = orc_bspline_sinc_sum(mz, in->nz, in->order, in->alias_extent);
  }
}

static void free_green(green_ctx *g) {
  free(g->dx); free(g->dy); free(g->dz); free(g->sx); free(g->sy); free(g->sz);
}

int orc_mesh_solve(const orc_mesh_in *in, orc_mesh_out *out) {
  const int nx = in->nx, ny = in->ny, nz = in->nz, p = in->order;
  const int nxh = nx / 2 + 1;
  const long ng = (long)nx * ny * nz, nh = (long)nz * ny * nxh;
  const int M = in->M;
  double ci[9], det;
  inv3(in->cell, ci, &det);
  const double vol = fabs(det);
  const double N3 = (double)ng;
  const double rho_scale = N3 / vol;

  /* ---- spread (serial, input order, as lmp/sog.cpp:1977-2018) ---- */
  double *rho = calloc(ng, sizeof(double));
  int c2d[3 * 216];
  if (in->spline == ORC_CUBES2) orc_cubes2_nodes(p, c2d, NULL);
  for (int i = 0; i < in->natoms && in->spline == ORC_CUBES2; ++i) {
    int i0[3];
    double w[216];
    const int nn = c2_stencil(p, ci, in->r + 3 * i, nx, ny, nz, i0, w);
    const double qs = rho_scale * in->q[i];
    for (int k = 0; k < nn; ++k) {
      const int gx = ((i0[0] + c2d[3 * k]) % nx + nx) % nx;
      const int gy = ((i0[1] + c2d[3 * k + 1]) % ny + ny) % ny;
      const int gz = ((i0[2] + c2d[3 * k + 2]) % nz + nz) % nz;
      rho[((long)gz * ny + gy) * nx + gx] += qs * w[k];
    }
  }
  for (int i = 0; i < in->natoms && in->spline != ORC_CUBES2; ++i) {
    int i0[3];
    double wx[8], wy[8], wz[8];
    atom_stencil(in->spline, p, ci, in->r + 3 * i, nx, ny, nz, i0, wx, wy, wz);
    const double qs = rho_scale * in->q[i];
    for (int c = 0; c < p; ++c) {
      const int gz = (i0[2] + c) % nz;
      for (int b = 0; b < p; ++b) {
        const int gy = (i0[1] + b) % ny;
        for (int a = 0; a < p; ++a) {
          const int gx = (i0[0] + a) % nx;
          rho[((long)gz * ny + gy) * nx + gx] += qs * wx[a] * wy[b] * wz[c];
        }
      }
    }
  }
  cplx *rk = malloc(sizeof(cplx) * nh);
  orc_rfft3(rho, rk, nx, ny, nz);
  free(rho);

  green_ctx g;
  setup_green(&g, in, ci);
  const int nf = in->want_force ? 3 : 0;
  const int want_phi = in->want_pot || in->want_dedr;   /* the potential field */
  const int nfield = nf + (want_phi ? 1 : 0);
  cplx *fields = nfield ? calloc(nh * nfield, sizeof(cplx)) : NULL;
  const double s2 = 1.0 / (N3 * N3);

  /* per-z-plane partial sums, combined serially: deterministic */
  const int nacc = 2 + 4 * M + 13;
  double *part = calloc((size_t)nz * nacc, sizeof(double));
#pragma omp parallel for schedule(static)
  for (int iz = 0; iz < nz; ++iz) {
    double *acc = part + (size_t)iz * nacc;
    double emD[64], emS[64], emDb[64], emSb[64];
    const int mz = iz <= nz / 2 ? iz : iz - nz;
    for (int iy = 0; iy < ny; ++iy) {
      const int my = iy <= ny / 2 ? iy : iy - ny;
      for (int mx = 0; mx < nxh; ++mx) {
        const long idx = ((long)iz * ny + iy) * nxh + mx;
        double k[3], K = 0, gE = 0, gF = 0, gS = 0, gV = 0, Kv = 0;
        const int live = green_at(&g, mx, my, mz, iy, iz, k, &K, &gE, &gF, &gS, &gV,
                                  &Kv, in->want_param_grad ? emD : NULL, emS, emDb, emSb);
        if (!live) continue;
        const double w = (mx == 0 || (nx % 2 == 0 && mx == nx / 2)) ? 1.0 : 2.0;
        const cplx r = rk[idx];
        const double r2 = r.re * r.re + r.im * r.im;
        acc[0] += w * gE * r2;
        acc[1] += w * gS;
        if (in->want_param_grad) {
          for (int m = 0; m < M; ++m) {
            acc[2 + m] += w * emD[m] * r2;
            acc[2 + M + m] += w * emS[m];
            acc[2 + 2 * M + m] += w * in->amp[m] * emDb[m] * r2;
            acc[2 + 3 * M + m] += w * in->amp[m] * emSb[m];
          }
        }
        if (in->want_virial) {
          double *v = acc + 2 + 4 * M;
          const double kk[6] = {k[0] * k[0], k[1] * k[1], k[2] * k[2],
                                k[0] * k[1], k[0] * k[2], k[1] * k[2]};
          v[0] += w * r2 * gE;
          for (int c = 0; c < 6; ++c) v[1 + c] += w * r2 * gV * kk[c];
          for (int c = 0; c < 6; ++c) v[7 + c] += w * Kv * kk[c];
        }
        if (nfield) {
          const double sre = gF * r.re / N3, sim = gF * r.im / N3;
          if (in->want_force) {
            for (int a = 0; a < 3; ++a) {
              fields[a * nh + idx].re = -k[a] * sim;
              fields[a * nh + idx].im = k[a] * sre;
            }
          }
          if (want_phi) {
            fields[nf * nh + idx].re = gE * r.re / N3;
            fields[nf * nh + idx].im = gE * r.im / N3;
          }
        }
      }
    }
  }
  double acc[2 + 4 * 64 + 13];
  memset(acc, 0, sizeof(double) * nacc);
  for (int iz = 0; iz < nz; ++iz)
    for (int c = 0; c < nacc; ++c) acc[c] += part[(size_t)iz * nacc + c];
  free(part);
  free(rk);

  double qsq = 0.0;
  for (int i = 0; i < in->natoms; ++i) qsq += in->q[i] * in->q[i];
  const double diag = acc[1] / (2.0 * vol);
  double e = 0.5 * vol * s2 * acc[0];
  if (in->remove_self) e -= qsq * diag;
  if (in->self_coeff != 0.0) e -= qsq * in->self_coeff;
  out->energy = e * in->norm_factor;
  out->diag_sum = diag;

  if (in->want_param_grad) {
    for (int m = 0; m < M; ++m) {
      double ga = 0.5 * vol * s2 * acc[2 + m];
      double gb = 0.5 * vol * s2 * acc[2 + 2 * M + m];
      if (in->remove_self) {
        ga -= qsq * acc[2 + M + m] / (2.0 * vol);
        gb -= qsq * acc[2 + 3 * M + m] / (2.0 * vol);
      }
      if (out->grad_amp) out->grad_amp[m] = ga * in->norm_factor;
      if (out->grad_bw2) out->grad_bw2[m] = gb * in->norm_factor;
    }
  }
  if (in->want_virial) {
    const double *v = acc + 2 + 4 * M;
    const double pref = in->norm_factor * 0.5 * vol * s2;
    const int comp[3][3] = {{0, 3, 4}, {3, 1, 5}, {4, 5, 2}};
    for (int a = 0; a < 3; ++a)
      for (int b = 0; b < 3; ++b) {
        double W = -pref * v[1 + comp[a][b]];
        if (a == b) W += pref * v[0];
        if (in->remove_self) {
          const double pv = qsq * in->norm_factor / (2.0 * vol);
          W += pv * v[7 + comp[a][b]];
          if (a == b) W -= qsq * in->norm_factor * diag;
        }
        out->virial[a * 3 + b] = W;
      }
  }

  if (nfield) {
    double *grids = malloc(sizeof(double) * ng * nfield);
    for (int f = 0; f < nfield; ++f) orc_irfft3(fields + f * nh, grids + f * ng, nx, ny, nz);
    free(fields);
#pragma omp parallel for schedule(static)
    for (int i = 0; i < in->natoms; ++i) {
      int i0[3];
      double wx[8], wy[8], wz[8];
      double accf[4] = {0, 0, 0, 0};
      if (in->spline == ORC_CUBES2) {
        double w[216];
        const int nn = c2_stencil(p, ci, in->r + 3 * i, nx, ny, nz, i0, w);
        for (int k = 0; k < nn; ++k) {
          const int gx = ((i0[0] + c2d[3 * k]) % nx + nx) % nx;
          const int gy = ((i0[1] + c2d[3 * k + 1]) % ny + ny) % ny;
          const int gz = ((i0[2] + c2d[3 * k + 2]) % nz + nz) % nz;
          const long idx = ((long)gz * ny + gy) * nx + gx;
          for (int f = 0; f < nfield; ++f) accf[f] += w[k] * grids[f * ng + idx];
        }
      } else {
      atom_stencil(in->spline, p, ci, in->r + 3 * i, nx, ny, nz, i0, wx, wy, wz);
      double dw[3][8], g3[3] = {0, 0, 0};
      if (in->want_dedr) {
        /* derivative weights d w / d t_a along each axis at the same t */
        const int n3[3] = {nx, ny, nz};
        for (int a = 0; a < 3; ++a) {
          double f = in->r[3 * i + 0] * ci[0 * 3 + a] + in->r[3 * i + 1] * ci[1 * 3 + a] +
                     in->r[3 * i + 2] * ci[2 * 3 + a];
          f = f - floor(f);
          const double fx = f * (double)n3[a];
          const double t = fx - floor(fx);
          if (in->spline == ORC_QUADS) orc_quads_dweights(p, t, dw[a]);
          else orc_bspline_dweights(p, t, dw[a]);
        }
      }
      for (int c = 0; c < p; ++c) {
        const int gz = (i0[2] + c) % nz;
        for (int b = 0; b < p; ++b) {
          const int gy = (i0[1] + b) % ny;
          for (int a = 0; a < p; ++a) {
            const int gx = (i0[0] + a) % nx;
            const long idx = ((long)gz * ny + gy) * nx + gx;
            const double w = wx[a] * wy[b] * wz[c];
            for (int f = 0; f < nfield; ++f) accf[f] += w * grids[f * ng + idx];
            if (in->want_dedr) {
              const double phi = grids[nf * ng + idx];
              g3[0] += dw[0][a] * wy[b] * wz[c] * phi;
              g3[1] += wx[a] * dw[1][b] * wz[c] * phi;
              g3[2] += wx[a] * wy[b] * dw[2][c] * phi;
            }
          }
        }
      }
      if (in->want_dedr) {
        /* t_a = n_a (r . cell^-1)_a + const: d t_a / d r_b = n_a ci[b][a] */
        const double n3d[3] = {(double)nx, (double)ny, (double)nz};
        for (int b = 0; b < 3; ++b) {
          double v = 0.0;
          for (int a = 0; a < 3; ++a) v += n3d[a] * ci[b * 3 + a] * g3[a];
          out->dedr[3 * i + b] = in->q[i] * v * in->norm_factor;
        }
      }
      }
      if (in->want_force)
        for (int a = 0; a < 3; ++a)
          out->forces[3 * i + a] = -in->q[i] * accf[a] * in->norm_factor;
      if (in->want_pot) {
        double v = accf[nf];
        if (in->remove_self) v -= 2.0 * in->q[i] * diag;
        if (in->self_coeff != 0.0) v -= 2.0 * in->q[i] * in->self_coeff;
        out->potential[i] = v * in->norm_factor;
      }
    }
    free(grids);
  }
  free_green(&g);
  return 0;
}

/* ------------------------------------------------------------------------ */
/* direct k-sum (gaussian.py:906-1081, 1281-1337), explicit derivatives      */
/* ------------------------------------------------------------------------ */

typedef struct {
  int natoms;
  const double *r, *q;
  double cell[9];
  int nk[3];
  int M;
  const double *amp, *bw2;
  double k_sq_max, norm_factor, self_coeff;
  int remove_self;
} orc_direct_in;

typedef struct {
  double energy, diag_sum;
  int nmodes_half;
  double *forces, *potential, *grad_amp, *grad_bw2;
} orc_direct_out;

int orc_direct_solve(const orc_direct_in *in, orc_direct_out *out) {
  double ci[9], det;
  inv3(in->cell, ci, &det);
  const double vol = fabs(det);
  const int N = in->natoms, M = in->M;
  const double tp = 2.0 * ORC_PI;
  double e_rec = 0.0, ksum = 0.0;
  double *ga = calloc(M, sizeof(double)), *gb = calloc(M, sizeof(double));
  double *ga_s = calloc(M, sizeof(double)), *gb_s = calloc(M, sizeof(double));
  double *fr = calloc((size_t)N * 3, sizeof(double)), *pot = calloc(N, sizeof(double));
  double *cs = malloc(sizeof(double) * N), *sn = malloc(sizeof(double) * N);
  int nmodes = 0;
  for (int n0 = 0; n0 <= in->nk[0]; ++n0)
    for (int n1 = -in->nk[1]; n1 <= in->nk[1]; ++n1)
      for (int n2 = -in->nk[2]; n2 <= in->nk[2]; ++n2) {
        /* half space: n0>0 | n0==0&n1>0 | n0==n1==0&n2>0 (gaussian.py:1318-1322
         * applies the same rule to the Cartesian k; for a right-handed cell the
         * pairing (k,-k) is the same set). */
        if (!(n0 > 0 || (n0 == 0 && n1 > 0) || (n0 == 0 && n1 == 0 && n2 > 0))) continue;
        double k[3];
        for (int a = 0; a < 3; ++a)
          k[a] = tp * (ci[a * 3 + 0] * n0 + ci[a * 3 + 1] * n1 + ci[a * 3 + 2] * n2);
        const double ksq = k[0] * k[0] + k[1] * k[1] + k[2] * k[2];
        if (ksq > in->k_sq_max) continue;
        ++nmodes;
        double K = 0.0;
        for (int m = 0; m < M; ++m) K += in->amp[m] * exp(-0.5 * in->bw2[m] * ksq);
        double sr = 0.0, si = 0.0;
        for (int i = 0; i < N; ++i) {
          const double kr = in->r[3 * i] * k[0] + in->r[3 * i + 1] * k[1] + in->r[3 * i + 2] * k[2];
          cs[i] = cos(kr); sn[i] = sin(kr);
          sr += in->q[i] * cs[i]; si += in->q[i] * sn[i];
        }
        const double s2 = sr * sr + si * si;
        e_rec += K * s2;
        ksum += K;
        for (int m = 0; m < M; ++m) {
          const double e = exp(-0.5 * in->bw2[m] * ksq);
          ga[m] += e * s2; ga_s[m] += e;
          gb[m] += -0.5 * ksq * in->amp[m] * e * s2;
          gb_s[m] += -0.5 * ksq * in->amp[m] * e;
        }
        for (int i = 0; i < N; ++i) {
          const double t = 2.0 * K * in->q[i] * (si * cs[i] - sr * sn[i]);
          fr[3 * i] += t * k[0]; fr[3 * i + 1] += t * k[1]; fr[3 * i + 2] += t * k[2];
          pot[i] += 2.0 * K * (sr * cs[i] + si * sn[i]);
        }
      }
  /* full sphere = 2 * half sphere; E = (1/2V) sum_full K |S|^2 */
  double qsq = 0.0;
  for (int i = 0; i < N; ++i) qsq += in->q[i] * in->q[i];
  const double diag = 2.0 * ksum / (2.0 * vol);
  double e = 2.0 * e_rec / (2.0 * vol);
  if (in->remove_self) e -= qsq * diag;
  if (in->self_coeff != 0.0) e -= qsq * in->self_coeff;
  out->energy = e * in->norm_factor;
  out->diag_sum = diag;
  out->nmodes_half = nmodes;
  for (int i = 0; i < N; ++i) {
    if (out->forces)
      for (int a = 0; a < 3; ++a) out->forces[3 * i + a] = -in->norm_factor * fr[3 * i + a] / vol;
    if (out->potential) {
      double v = pot[i] / vol;
      if (in->remove_self) v -= 2.0 * in->q[i] * diag;
      if (in->self_coeff != 0.0) v -= 2.0 * in->q[i] * in->self_coeff;
      out->potential[i] = v * in->norm_factor;
    }
  }
  for (int m = 0; m < M; ++m) {
    double a = ga[m] / vol, b = gb[m] / vol;
    if (in->remove_self) { a -= qsq * ga_s[m] / vol; b -= qsq * gb_s[m] / vol; }
    if (out->grad_amp) out->grad_amp[m] = a * in->norm_factor;
    if (out->grad_bw2) out->grad_bw2[m] = b * in->norm_factor;
  }
  free(ga); free(gb); free(ga_s); free(gb_s); free(fr); free(pot); free(cs); free(sn);
  return 0;
}

int orc_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* threads of the following parallel regions (a launcher's OMP_NUM_THREADS=1
   would otherwise leave the timed CPU baseline on one core) */
void orc_set_num_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

/* ------------------------------------------------------------------------ */
/* real-space pair sum (non-periodic frames)                                */
/* ------------------------------------------------------------------------ */

/* One non-periodic frame, all channels (compute_potential_realspace,
 * src/sog/module/gaussian.py:822-845):
 *   E = norm * ( 1/2 sum_{i != j} (q_i . q_j) sum_m amp_m exp(-r_ij^2 / (2 bw2_m))
 *                + [!remove_self] 1/2 sum_i |q_i|^2 sum_m amp_m )
 * q is [n, C] row-major.  Explicit derivatives (the reference takes them by
 * autograd): forces [n,3], dE/dq [n,C], dE/damp [M], dE/dbw2 [M]; any output
 * pointer may be NULL.  Returns the energy. */
double orc_realspace_solve(int n, int C, const double *r, const double *q, int M, const double *amp,
                           const double *bw2, double norm_factor, int remove_self, double *forces,
                           double *potential, double *grad_amp, double *grad_bw2) {
  double e_pair = 0.0;
  double *ga = calloc((size_t)M, sizeof(double)), *gb = calloc((size_t)M, sizeof(double));
#pragma omp parallel
  {
    double *ga_t = calloc((size_t)M, sizeof(double)), *gb_t = calloc((size_t)M, sizeof(double));
    double *ex = malloc(sizeof(double) * (size_t)M);
    double e_t = 0.0;
#pragma omp for schedule(static)
    for (int i = 0; i < n; ++i) {
      double f[3] = {0.0, 0.0, 0.0};
      double pi[8] = {0.0};
      double *pv = C <= 8 ? pi : calloc((size_t)C, sizeof(double));
      for (int j = 0; j < n; ++j) {
        if (j == i) continue;
        const double dx = r[3 * i] - r[3 * j], dy = r[3 * i + 1] - r[3 * j + 1], dz = r[3 * i + 2] - r[3 * j + 2];
        const double r2 = dx * dx + dy * dy + dz * dz;
        double K = 0.0, Kd = 0.0, qq = 0.0;
        for (int m = 0; m < M; ++m) {
          ex[m] = exp(-0.5 * r2 / bw2[m]);
          K += amp[m] * ex[m];
          Kd += amp[m] * ex[m] / bw2[m];
        }
        for (int c = 0; c < C; ++c) {
          qq += q[(size_t)i * C + c] * q[(size_t)j * C + c];
          pv[c] += K * q[(size_t)j * C + c];
        }
        /* d/dr_i of 1/2 sum_{a != b} qq K(r_ab^2) = -sum_j qq Kd (r_i - r_j) */
        f[0] += qq * Kd * dx; f[1] += qq * Kd * dy; f[2] += qq * Kd * dz;
        e_t += 0.5 * qq * K;
        for (int m = 0; m < M; ++m) {
          ga_t[m] += 0.5 * qq * ex[m];
          gb_t[m] += 0.5 * qq * amp[m] * ex[m] * 0.5 * r2 / (bw2[m] * bw2[m]);
        }
      }
      if (forces)
        for (int a = 0; a < 3; ++a) forces[3 * i + a] = norm_factor * f[a];
      if (potential)
        for (int c = 0; c < C; ++c) potential[(size_t)i * C + c] = norm_factor * pv[c];
      if (pv != pi) free(pv);
    }
#pragma omp critical
    {
      e_pair += e_t;
      for (int m = 0; m < M; ++m) { ga[m] += ga_t[m]; gb[m] += gb_t[m]; }
    }
    free(ga_t); free(gb_t); free(ex);
  }
  double e = e_pair;
  double qsq = 0.0, asum = 0.0;
  for (size_t k = 0; k < (size_t)n * C; ++k) qsq += q[k] * q[k];
  for (int m = 0; m < M; ++m) asum += amp[m];
  if (!remove_self) {
    e += 0.5 * qsq * asum;
    if (potential)
      for (size_t k = 0; k < (size_t)n * C; ++k) potential[k] += norm_factor * q[k] * asum;
  }
  for (int m = 0; m < M; ++m) {
    if (grad_amp) grad_amp[m] = norm_factor * (ga[m] + (remove_self ? 0.0 : 0.5 * qsq));
    if (grad_bw2) grad_bw2[m] = norm_factor * gb[m];
  }
  free(ga); free(gb);
  return e * norm_factor;
}
