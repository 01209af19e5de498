/*
 * CPU port of the SSIM forward + backward -- TEST INFRASTRUCTURE (the timed
 * CPU baseline of bench.py for the fwd+bwd path), not product code.
 *
 * The reference's CPU library (frame_analytics/csrc/fa_cpu.cpp) has a forward
 * only; its training path runs torch autograd.  This file restates, in
 * float64 C threaded over planes, the forward of reference.py:118-160 and the
 * backward of fa_cuda.cu:551-607 (coefficient maps) + 655-784 (transposed
 * blur), so the fwd+bwd step has a CPU number measured on the same host.
 *
 *   ssim_port_fwd_bwd(x, y, planes, H, W, win, K, C1, C2, g, out_s, dx, dy)
 *     x, y   : float32 [planes][H][W]
 *     g      : upstream gradient for every map position (e.g. -1/(P*Hout*Wout))
 *     out_s  : [planes] sum of the SSIM map
 *     dx, dy : float32 [planes][H][W] (either may be NULL)
 */
#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
  const float *x, *y;
  int planes, H, W, K;
  double w[16];
  double C1, C2, g;
  double* out_s;
  float *dx, *dy;
  int next;
  pthread_mutex_t mu;
} job_t;

/* valid separable blur of an H x W double image -> Ho x Wo */
static void blur_valid(const double* in, int H, int W, const double* w, int K, double* tmp,
                       double* out) {
  const int Wo = W - K + 1, Ho = H - K + 1;
  for (int r = 0; r < H; ++r) {
    const double* a = in + (size_t)r * W;
    double* t = tmp + (size_t)r * Wo;
    for (int c = 0; c < Wo; ++c) {
      double s = 0.0;
      for (int j = 0; j < K; ++j) s += w[j] * a[c + j];
      t[c] = s;
    }
  }
  for (int r = 0; r < Ho; ++r) {
    double* o = out + (size_t)r * Wo;
    for (int c = 0; c < Wo; ++c) o[c] = 0.0;
    for (int i = 0; i < K; ++i) {
      const double* t = tmp + (size_t)(r + i) * Wo;
      for (int c = 0; c < Wo; ++c) o[c] += w[i] * t[c];
    }
  }
}

/* adjoint of blur_valid: Ho x Wo -> H x W (zeros outside the valid grid) */
static void blur_full_t(const double* in, int H, int W, const double* w, int K, double* tmp,
                        double* out) {
  const int Wo = W - K + 1, Ho = H - K + 1;
  memset(tmp, 0, sizeof(double) * (size_t)H * Wo);
  for (int r = 0; r < Ho; ++r)
    for (int i = 0; i < K; ++i) {
      double* t = tmp + (size_t)(r + i) * Wo;
      const double* a = in + (size_t)r * Wo;
      for (int c = 0; c < Wo; ++c) t[c] += w[i] * a[c];
    }
  memset(out, 0, sizeof(double) * (size_t)H * W);
  for (int r = 0; r < H; ++r) {
    const double* t = tmp + (size_t)r * Wo;
    double* o = out + (size_t)r * W;
    for (int c = 0; c < Wo; ++c)
      for (int j = 0; j < K; ++j) o[c + j] += w[j] * t[c];
  }
}

static void plane(job_t* J, int p, double* buf) {
  const int H = J->H, W = J->W, K = J->K, Ho = H - K + 1, Wo = W - K + 1;
  const size_t n = (size_t)H * W, no = (size_t)Ho * Wo;
  double *X = buf, *Y = X + n, *T = Y + n, *tmp = T + n;
  double *mx = tmp + n, *my = mx + no, *exx = my + no, *eyy = exx + no, *exy = eyy + no;
  const float* xs = J->x + (size_t)p * n;
  const float* ys = J->y + (size_t)p * n;
  for (size_t i = 0; i < n; ++i) { X[i] = xs[i]; Y[i] = ys[i]; }
  blur_valid(X, H, W, J->w, K, tmp, mx);
  blur_valid(Y, H, W, J->w, K, tmp, my);
  for (size_t i = 0; i < n; ++i) T[i] = X[i] * X[i];
  blur_valid(T, H, W, J->w, K, tmp, exx);
  for (size_t i = 0; i < n; ++i) T[i] = Y[i] * Y[i];
  blur_valid(T, H, W, J->w, K, tmp, eyy);
  for (size_t i = 0; i < n; ++i) T[i] = X[i] * Y[i];
  blur_valid(T, H, W, J->w, K, tmp, exy);
  double ssum = 0.0;
  /* reuse the moment planes for the coefficients b, c, tx, ty */
  for (size_t i = 0; i < no; ++i) {
    const double ux = mx[i], uy = my[i];
    const double sxx = exx[i] - ux * ux, syy = eyy[i] - uy * uy, sxy = exy[i] - ux * uy;
    const double A1 = 2 * ux * uy + J->C1, A2 = 2 * sxy + J->C2;
    const double B1 = ux * ux + uy * uy + J->C1, B2 = sxx + syy + J->C2;
    const double S = A1 * A2 / (B1 * B2);
    ssum += S;
    const double g = J->g;
    const double b = g * (-S / B2), c = g * (2 * A1 / (B1 * B2));
    const double k = g * 2 * A2 / (B1 * B2);
    const double tx = k * (uy - ux * A1 / B1) - 2 * b * ux - c * uy;
    const double ty = k * (ux - uy * A1 / B1) - 2 * b * uy - c * ux;
    mx[i] = b; my[i] = c; exx[i] = tx; eyy[i] = ty;
  }
  J->out_s[p] = ssum;
  double *Pb = T, *Pc = buf + 9 * n, *Pt = Pc + n; /* 11n of the 12n doubles */
  blur_full_t(mx, H, W, J->w, K, tmp, Pb);
  blur_full_t(my, H, W, J->w, K, tmp, Pc);
  if (J->dx) {
    blur_full_t(exx, H, W, J->w, K, tmp, Pt);
    float* o = J->dx + (size_t)p * n;
    for (size_t i = 0; i < n; ++i) o[i] = (float)(2 * X[i] * Pb[i] + Y[i] * Pc[i] + Pt[i]);
  }
  if (J->dy) {
    blur_full_t(eyy, H, W, J->w, K, tmp, Pt);
    float* o = J->dy + (size_t)p * n;
    for (size_t i = 0; i < n; ++i) o[i] = (float)(2 * Y[i] * Pb[i] + X[i] * Pc[i] + Pt[i]);
  }
}

static void* worker(void* arg) {
  job_t* J = (job_t*)arg;
  const size_t n = (size_t)J->H * J->W;
  double* buf = (double*)malloc(sizeof(double) * 12 * n);
  if (!buf) return NULL;
  for (;;) {
    pthread_mutex_lock(&J->mu);
    const int p = J->next++;
    pthread_mutex_unlock(&J->mu);
    if (p >= J->planes) break;
    plane(J, p, buf);
  }
  free(buf);
  return NULL;
}

int ssim_port_fwd_bwd(const float* x, const float* y, int planes, int H, int W,
                      const double* win, int K, double C1, double C2, double g, double* out_s,
                      float* dx, float* dy, int threads) {
  if (K > 15 || H < K || W < K || threads < 1) return 2;
  job_t J;
  memset(&J, 0, sizeof(J));
  J.x = x; J.y = y; J.planes = planes; J.H = H; J.W = W; J.K = K;
  for (int i = 0; i < K; ++i) J.w[i] = win[i];
  J.C1 = C1; J.C2 = C2; J.g = g; J.out_s = out_s; J.dx = dx; J.dy = dy;
  pthread_mutex_init(&J.mu, NULL);
  if (threads > planes) threads = planes;
  pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * threads);
  for (int t = 0; t < threads; ++t) pthread_create(&th[t], NULL, worker, &J);
  for (int t = 0; t < threads; ++t) pthread_join(th[t], NULL);
  free(th);
  pthread_mutex_destroy(&J.mu);
  return 0;
}
