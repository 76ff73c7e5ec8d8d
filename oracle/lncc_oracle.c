/*
 * TEST INFRASTRUCTURE ONLY - the CPU oracle for the fused LNCC loss. Nothing in the product links,
 * loads or calls this file; tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use it
 * as the checker.
 *
 * An fp64 restatement of the reference algorithm with the reference CUDA kernel's semantics:
 *  - box sums over the k^3 window, zero padded, n = k^3 everywhere (fused_lncc/csrc/lncc3d.cu:44-53,93)
 *  - cross = Spt - Sp*St/n; var = max(Sxx - Sx^2/n, 0) + dr            (lncc3d.cu:93-97)
 *  - cc = cross^2/(var_p*var_t); cc >= 1 -> 1 with zero adjoints; NaN stays NaN with zero
 *    adjoints                                                            (lncc3d.cu:98-107)
 *  - adjoints Cc = 2 cross/(vp vt), Bc = -cross^2/(vp^2 vt), A = -(St Cc + 2 Sp Bc)/n (lncc3d.cu:101-104)
 *  - d(sum cc)/dp = box(A) + 2 p box(Bc) + t box(Cc)                     (lncc3d.cu:163,231-233)
 *  - loss = 1 - mean(cc)                                                 (fused_lncc/__init__.py:62)
 * The PyTorch oracle of the reference (baselines/torch_lncc.py:25-32) is the same formula without
 * the max(.,0) clamp; the two agree wherever var >= 0, which holds on the golden vectors.
 *
 * Separable running sums in double precision; planes parallelised with OpenMP.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* y = zero-padded box of half-width r along one axis of a (n0, n1, n2) array (axis 0, 1 or 2). */
static void box_axis(const double* x, double* y, int64_t n0, int64_t n1, int64_t n2, int axis, int r) {
  int64_t len, stride, nlines;
  if (axis == 2) { len = n2; stride = 1; nlines = n0 * n1; }
  else if (axis == 1) { len = n1; stride = n2; nlines = n0 * n2; }
  else { len = n0; stride = n1 * n2; nlines = n1 * n2; }
#pragma omp parallel for schedule(static)
  for (int64_t l = 0; l < nlines; ++l) {
    int64_t base;
    if (axis == 2) base = l * n2;
    else if (axis == 1) base = (l / n2) * n1 * n2 + (l % n2);
    else base = l;
    /* prefix sums in a local buffer, then window differences */
    double* pre = (double*)malloc(sizeof(double) * (size_t)(len + 1));
    pre[0] = 0.0;
    for (int64_t i = 0; i < len; ++i) pre[i + 1] = pre[i] + x[base + i * stride];
    for (int64_t i = 0; i < len; ++i) {
      int64_t lo = i - r, hi = i + r + 1;
      if (lo < 0) lo = 0;
      if (hi > len) hi = len;
      y[base + i * stride] = pre[hi] - pre[lo];
    }
    free(pre);
  }
}

/* Half-widths of the window along D, H, W (a cubic window has rd = rh = rw = k/2). */
typedef struct { int rd, rh, rw; } Radii;

static void box3(const double* x, double* y, double* tmp, int64_t D, int64_t H, int64_t W, Radii r) {
  box_axis(x, y, D, H, W, 2, r.rw);
  box_axis(y, tmp, D, H, W, 1, r.rh);
  box_axis(tmp, y, D, H, W, 0, r.rd);
}

/* Direct (non-prefix) box for accuracy on the golden vectors: sum of the window, in double. */
static void box3_direct(const double* x, double* y, double* tmp, int64_t D, int64_t H, int64_t W, Radii rr) {
  const int64_t HW = H * W;
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < D * HW; ++i) {
    int64_t w = i % W, h = (i / W) % H, z = i / HW;
    (void)z; (void)h;
    double s = 0.0;
    for (int64_t d = -rr.rw; d <= rr.rw; ++d) {
      int64_t ww = w + d;
      if (ww >= 0 && ww < W) s += x[i + d];
    }
    tmp[i] = s;
  }
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < D * HW; ++i) {
    int64_t h = (i / W) % H;
    double s = 0.0;
    for (int64_t d = -rr.rh; d <= rr.rh; ++d) {
      int64_t hh = h + d;
      if (hh >= 0 && hh < H) s += tmp[i + d * W];
    }
    y[i] = s;
  }
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < D * HW; ++i) {
    int64_t z = i / HW;
    double s = 0.0;
    for (int64_t d = -rr.rd; d <= rr.rd; ++d) {
      int64_t zz = z + d;
      if (zz >= 0 && zz < D) s += y[i + d * HW];
    }
    tmp[i] = s;
  }
  memcpy(y, tmp, sizeof(double) * (size_t)(D * HW));
}

static void do_box(int direct, const double* x, double* y, double* tmp, int64_t D, int64_t H, int64_t W,
                   Radii r) {
  if (direct) box3_direct(x, y, tmp, D, H, W, r);
  else box3(x, y, tmp, D, H, W, r);
}

/*
 * Loss / gradient / maps for B volumes of (D,H,W), fp32 in, fp64 math.
 *   z_begin, z_end : output planes (loss terms, grad planes), as in lncc_fused_forward.
 *   cc_sum         : out, sum of cc over the output planes (all volumes).
 *   grad           : NULL or (B, z_end-z_begin, H, W) fp32 receiving grad_scale * d(sum cc)/dp.
 *   ncc, A, Bc, Cc : NULL or (B, D, H, W) fp32 maps as the reference lncc_forward returns them
 *                    (lncc3d.cu:108: ncc clamped map and the three unscaled adjoints).
 *   direct         : 1 = direct window sums, 0 = prefix-sum differences (faster).
 * Returns 0, or -1 on bad arguments / allocation failure.
 */
/*
 * As oracle_lncc for a kd x kh x kw window (each side odd): the same math with n = kd*kh*kw. The
 * reference has cubic windows only; this serves the non-cubic windows its roadmap lists as open
 * (BENCHMARKS.md:177-178).
 */
int oracle_lncc_win(const float* p, const float* t, int64_t B, int64_t D, int64_t H, int64_t W, int kd, int kh,
                    int kw, double dr, int64_t z_begin, int64_t z_end, double* cc_sum, float* grad,
                    double grad_scale, float* ncc, float* A_out, float* B_out, float* C_out, int direct) {
  if (!p || !t || B < 1 || D < 1 || H < 1 || W < 1) return -1;
  if (kd < 1 || kh < 1 || kw < 1 || (kd % 2) == 0 || (kh % 2) == 0 || (kw % 2) == 0) return -1;
  if (z_begin < 0 || z_end > D || z_end <= z_begin) return -1;
  const Radii r = {kd / 2, kh / 2, kw / 2};
  const double n = (double)kd * kh * kw;
  const int64_t V = D * H * W, HW = H * W;
  double* f[5];
  double* adj[3];
  double* tmp = (double*)malloc(sizeof(double) * (size_t)V);
  double* raw = (double*)malloc(sizeof(double) * (size_t)V);
  int ok = tmp && raw;
  for (int i = 0; i < 5; ++i) { f[i] = (double*)malloc(sizeof(double) * (size_t)V); ok = ok && f[i]; }
  for (int i = 0; i < 3; ++i) { adj[i] = (double*)malloc(sizeof(double) * (size_t)V); ok = ok && adj[i]; }
  double total = 0.0;
  if (ok) {
    for (int64_t b = 0; b < B; ++b) {
      const float* pb = p + b * V;
      const float* tb = t + b * V;
      for (int fi = 0; fi < 5; ++fi) {
#pragma omp parallel for schedule(static)
        for (int64_t i = 0; i < V; ++i) {
          const double pv = pb[i], tv = tb[i];
          raw[i] = fi == 0 ? pv : fi == 1 ? tv : fi == 2 ? pv * pv : fi == 3 ? tv * tv : pv * tv;
        }
        do_box(direct, raw, f[fi], tmp, D, H, W, r);
      }
      double vsum = 0.0;
#pragma omp parallel for schedule(static) reduction(+ : vsum)
      for (int64_t i = 0; i < V; ++i) {
        const double Sp = f[0][i], St = f[1][i], Spp = f[2][i], Stt = f[3][i], Spt = f[4][i];
        const double cross = Spt - Sp * St / n;
        double vp = Spp - Sp * Sp / n;
        double vt = Stt - St * St / n;
        vp = (vp > 0.0 ? vp : 0.0) + dr;
        vt = (vt > 0.0 ? vt : 0.0) + dr;
        double cc = (cross * cross) / (vp * vt);
        double a = 0.0, bb = 0.0, c = 0.0;
        if (cc < 1.0) {
          c = 2.0 * cross / (vp * vt);
          bb = -(cross * cross) / (vp * vp * vt);
          a = -(St * c + 2.0 * Sp * bb) / n;
        } else if (cc >= 1.0) {
          cc = 1.0;
        } /* NaN: cc stays NaN, adjoints zero */
        adj[0][i] = a;
        adj[1][i] = bb;
        adj[2][i] = c;
        const int64_t z = i / HW;
        if (z >= z_begin && z < z_end) vsum += cc;
        if (ncc) ncc[b * V + i] = (float)cc;
        if (A_out) A_out[b * V + i] = (float)a;
        if (B_out) B_out[b * V + i] = (float)bb;
        if (C_out) C_out[b * V + i] = (float)c;
      }
      total += vsum;
      if (grad) {
        for (int ai = 0; ai < 3; ++ai) {
          memcpy(raw, adj[ai], sizeof(double) * (size_t)V);
          do_box(direct, raw, adj[ai], tmp, D, H, W, r);
        }
        const int64_t nz = z_end - z_begin;
        float* gb = grad + b * nz * HW;
#pragma omp parallel for schedule(static)
        for (int64_t i = z_begin * HW; i < z_end * HW; ++i) {
          const double g = adj[0][i] + 2.0 * (double)pb[i] * adj[1][i] + (double)tb[i] * adj[2][i];
          gb[i - z_begin * HW] = (float)(grad_scale * g);
        }
      }
    }
  }
  if (cc_sum) *cc_sum = total;
  for (int i = 0; i < 5; ++i) free(f[i]);
  for (int i = 0; i < 3; ++i) free(adj[i]);
  free(tmp);
  free(raw);
  return ok ? 0 : -1;
}

int oracle_lncc(const float* p, const float* t, int64_t B, int64_t D, int64_t H, int64_t W, int k,
                double dr, int64_t z_begin, int64_t z_end, double* cc_sum, float* grad, double grad_scale,
                float* ncc, float* A_out, float* B_out, float* C_out, int direct) {
  return oracle_lncc_win(p, t, B, D, H, W, k, k, k, dr, z_begin, z_end, cc_sum, grad, grad_scale, ncc, A_out,
                         B_out, C_out, direct);
}

/* Zero-padded k^3 box sum of one fp32 field (reference box3d_sep_forward, lncc3d.cu:287-344). */
int oracle_box3d(const float* x, float* y, int64_t B, int64_t D, int64_t H, int64_t W, int k) {
  if (!x || !y || B < 1 || D < 1 || H < 1 || W < 1 || k < 1 || (k % 2) == 0) return -1;
  const int64_t V = D * H * W;
  double* a = (double*)malloc(sizeof(double) * (size_t)V);
  double* o = (double*)malloc(sizeof(double) * (size_t)V);
  double* tmp = (double*)malloc(sizeof(double) * (size_t)V);
  if (!a || !o || !tmp) { free(a); free(o); free(tmp); return -1; }
  for (int64_t b = 0; b < B; ++b) {
    for (int64_t i = 0; i < V; ++i) a[i] = x[b * V + i];
    const Radii rr = {k / 2, k / 2, k / 2};
    box3_direct(a, o, tmp, D, H, W, rr);
    for (int64_t i = 0; i < V; ++i) y[b * V + i] = (float)o[i];
  }
  free(a); free(o); free(tmp);
  return 0;
}

int oracle_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
