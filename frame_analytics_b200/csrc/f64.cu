// float64 SSIM, MS-SSIM pooling and GMSD on sm_100a: the metrics of float64
// frames computed in float64 throughout.
//
// The reference computes float64 input on its float64 torch path (its native
// kernels decline float64: frame_analytics/backend.py:466, 602); the float32
// kernels of this library would round such input to float32 first, which a
// pair that differs only below float32 resolution cannot survive.  These
// kernels keep every sum, moment and gradient in double.  They favour
// simplicity over speed (float64 frames are the exception on this path):
//
//   * ssim64_kernel: one block per 32 x 8 output tile of a plane.  The
//     (8 + K - 1) x (32 + K - 1) input tile of x and y is loaded (any strides,
//     luma folded in) into shared memory; a horizontal pass forms the five
//     blurred moments E[x], E[y], E[x^2], E[y^2], E[xy] of every tile row and a
//     vertical pass the output's SSIM and cs (reference.py:118-160).  In
//     coefficient mode it writes, per output position, the four backward
//     coefficient planes instead of SSIM sums;
//   * ssim64_scatter_kernel: dx = 2x (W'*b) + y (W'*c) + W'*tx and dy likewise
//     (W' the transposed, zero-padded window), from those planes;
//   * pool64_kernel / pool64_bwd_kernel: 2x2 average pool for the MS-SSIM
//     pyramid and its adjoint;
//   * gmsd64_kernel (statistics, or in coefficient mode dL/d(gradients) per
//     map position) and gmsd64_scatter_kernel: GMS map statistics and the
//     gradient of (mean, std) of q.
// Reductions use per-block partials and a last-block finaliser, as elsewhere.
#include <algorithm>

#include "common.cuh"

namespace fab {

constexpr int T64_W = 32, T64_H = 8;  // output tile
constexpr int T64_THREADS = T64_W * T64_H;
constexpr int MAXK = 11;

struct Ssim64Args {
  const char* x;
  const char* y;
  long long sn, sc, sh;
  int N, C, H, W;  // input planes (C = 3 with luma)
  int Cm, P;       // planes the metric sees
  int Hout, Wout, K;
  double w[MAXK];
  double C1, C2;
  double lk0, lk1, lk2, lk3;
  int luma;
  int tiles_x, tiles_y;
  // forward
  unsigned int* counter;
  double* part_s;   // [P][tiles]
  double* part_cs;  // [P][tiles] or null
  double* map;      // [P][Hout][Wout] or null
  double* out_plane_s;
  double* out_plane_cs;
  double* out_per_image;
  double* out_total;
  // coefficients (backward)
  int gmode;             // 0 map, 1 scalar, 2 per plane (s, cs)
  const double* dmap;    // [P][Hout][Wout]
  const double* gscalar; // [1]
  const double* gs;      // [P]
  const double* gcs;     // [P]
  double grad_norm;
  double* coef;          // [4][P][Hout][Wout]: b, c, tx, ty
};

template <typename T>
__device__ __forceinline__ double ld64(const char* base, long long o) {
  return Ld<T>::d(ldro(reinterpret_cast<const T*>(base) + o));
}

// Input sample (plane pl, row r, column c) in double, luma projected.
template <typename T>
__device__ __forceinline__ double px64(const Ssim64Args& p, const char* base, int pl, int r,
                                       int c) {
  const int n = pl / p.Cm, ch = pl - n * p.Cm;
  const long long o = (long long)n * p.sn + (long long)r * p.sh + c;
  if (p.luma) {
    return fma(p.lk0, ld64<T>(base, o), fma(p.lk1, ld64<T>(base, o + p.sc),
               fma(p.lk2, ld64<T>(base, o + 2 * p.sc), p.lk3)));
  }
  return ld64<T>(base, o + (long long)ch * p.sc);
}

// COEF = false: SSIM (and cs) sums + map; true: backward coefficient planes.
template <typename T, bool COEF>
__global__ void __launch_bounds__(T64_THREADS) ssim64_kernel(const Ssim64Args p) {
  constexpr int IW = T64_W + MAXK - 1, IH = T64_H + MAXK - 1;
  __shared__ double sx[IH][IW], sy[IH][IW];
  __shared__ double hm[5][IH][T64_W];
  __shared__ double s_red[32];
  __shared__ int s_flag;
  const int t = threadIdx.x, tx = t % T64_W, ty = t / T64_W;
  const int pl = blockIdx.z;
  const int ox0 = blockIdx.x * T64_W, oy0 = blockIdx.y * T64_H;
  const int K = p.K;
  const int ih = T64_H + K - 1, iw = T64_W + K - 1;
  for (int i = t; i < ih * iw; i += T64_THREADS) {
    const int r = i / iw, c = i - r * iw;
    const int gr = oy0 + r, gc = ox0 + c;
    const bool in = gr < p.H && gc < p.W;
    sx[r][c] = in ? px64<T>(p, p.x, pl, gr, gc) : 0.0;
    sy[r][c] = in ? px64<T>(p, p.y, pl, gr, gc) : 0.0;
  }
  __syncthreads();
  for (int i = t; i < ih * T64_W; i += T64_THREADS) {
    const int r = i / T64_W, c = i - r * T64_W;
    double a = 0, b = 0, aa = 0, bb = 0, ab = 0;
    for (int j = 0; j < K; ++j) {
      const double w = p.w[j], u = sx[r][c + j], v = sy[r][c + j];
      a = fma(w, u, a);
      b = fma(w, v, b);
      aa = fma(w, u * u, aa);
      bb = fma(w, v * v, bb);
      ab = fma(w, u * v, ab);
    }
    hm[0][r][c] = a; hm[1][r][c] = b; hm[2][r][c] = aa; hm[3][r][c] = bb; hm[4][r][c] = ab;
  }
  __syncthreads();
  const int oy = oy0 + ty, ox = ox0 + tx;
  const bool ok = oy < p.Hout && ox < p.Wout;
  double s = 0.0, cs = 0.0;
  if (ok) {
    double m[5] = {0, 0, 0, 0, 0};
    for (int j = 0; j < K; ++j) {
      const double w = p.w[j];
#pragma unroll
      for (int q = 0; q < 5; ++q) m[q] = fma(w, hm[q][ty + j][tx], m[q]);
    }
    const double mx = m[0], my = m[1];
    const double sxx = m[2] - mx * mx, syy = m[3] - my * my, sxy = m[4] - mx * my;
    const double A1 = 2 * mx * my + p.C1, A2 = 2 * sxy + p.C2;
    const double B1 = mx * mx + my * my + p.C1, B2 = sxx + syy + p.C2;
    const double S = (A1 * A2) / (B1 * B2);
    const long long o = ((long long)pl * p.Hout + oy) * p.Wout + ox;
    if constexpr (!COEF) {
      s = S;
      cs = A2 / B2;
      if (p.map) p.map[o] = S;
    } else {
      double g, gcs = 0.0;
      if (p.gmode == 0) g = p.dmap[o];
      else if (p.gmode == 1) g = p.gscalar[0] * p.grad_norm;
      else { g = p.gs[pl] * p.grad_norm; gcs = p.gcs[pl] * p.grad_norm; }
      const double CS = A2 / B2;
      const double b = -(g * S + gcs * CS) / B2;               // d/dsxx (= d/dsyy)
      const double c = 2.0 * (g * A1 / B1 + gcs) / B2;         // d/dsxy
      const double k = g * 2.0 * A2 / (B1 * B2);
      const double tx_ = k * (my - mx * A1 / B1) - 2 * b * mx - c * my;
      const double ty_ = k * (mx - my * A1 / B1) - 2 * b * my - c * mx;
      const long long plane = (long long)p.P * p.Hout * p.Wout;
      p.coef[o] = b;
      p.coef[o + plane] = c;
      p.coef[o + 2 * plane] = tx_;
      p.coef[o + 3 * plane] = ty_;
    }
  }
  if constexpr (!COEF) {
    const int tiles = p.tiles_x * p.tiles_y;
    const long long pidx = (long long)pl * tiles + blockIdx.y * p.tiles_x + blockIdx.x;
    s = block_sum(s, s_red);
    if (t == 0) p.part_s[pidx] = s;
    if (p.part_cs) {
      cs = block_sum(cs, s_red);
      if (t == 0) p.part_cs[pidx] = cs;
    }
    if (last_block_arrived(p.counter, gridDim.x * gridDim.y * gridDim.z, &s_flag)) {
      const double npix = (double)p.Hout * p.Wout;
      const int lane = t & 31, wid = t >> 5;
      for (int q = wid; q < p.P; q += T64_THREADS / 32) {
        double a = 0.0, b = 0.0;
        for (int i = lane; i < tiles; i += 32) {
          a += p.part_s[(long long)q * tiles + i];
          if (p.part_cs) b += p.part_cs[(long long)q * tiles + i];
        }
        a = warp_sum(a);
        b = warp_sum(b);
        if (lane == 0) {
          p.part_s[(long long)q * tiles] = a;
          if (p.out_plane_s) p.out_plane_s[q] = a / npix;
          if (p.out_plane_cs) p.out_plane_cs[q] = b / npix;
        }
      }
      __syncthreads();
      __threadfence_block();
      double tot = 0.0;
      for (int n = t; n < p.N; n += T64_THREADS) {
        double v = 0.0;
        for (int c = 0; c < p.Cm; ++c) v += p.part_s[(long long)(n * p.Cm + c) * tiles];
        if (p.out_per_image) p.out_per_image[n] = v / (npix * p.Cm);
        tot += v;
      }
      tot = block_sum(tot, s_red);
      if (t == 0 && p.out_total) *p.out_total = tot / (npix * p.P);
    }
  }
}

// Transposed blur of the coefficient planes: a tile of 32 x 8 input pixels
// needs coefficients at output rows/cols [i - K + 1, i], zero outside.
__global__ void __launch_bounds__(T64_THREADS) ssim64_scatter_kernel(const Ssim64Args p,
                                                                     const double* x,
                                                                     const double* y,
                                                                     double* dx, double* dy) {
  constexpr int IW = T64_W + MAXK - 1, IH = T64_H + MAXK - 1;
  __shared__ double sc[4][IH][IW];
  __shared__ double hs[4][IH][T64_W];
  const int t = threadIdx.x, tx = t % T64_W, ty = t / T64_W;
  const int pl = blockIdx.z;
  const int ix0 = blockIdx.x * T64_W, iy0 = blockIdx.y * T64_H;
  const int K = p.K;
  const int ch = T64_H + K - 1, cw = T64_W + K - 1;
  const long long plane = (long long)p.P * p.Hout * p.Wout;
  for (int i = t; i < ch * cw; i += T64_THREADS) {
    const int r = i / cw, c = i - r * cw;
    const int orow = iy0 - (K - 1) + r, ocol = ix0 - (K - 1) + c;
    const bool in = orow >= 0 && orow < p.Hout && ocol >= 0 && ocol < p.Wout;
    const long long o = ((long long)pl * p.Hout + orow) * p.Wout + ocol;
#pragma unroll
    for (int q = 0; q < 4; ++q) sc[q][r][c] = in ? p.coef[o + q * plane] : 0.0;
  }
  __syncthreads();
  // input column ix0 + c gathers output columns ix0 + c - j with tap j
  for (int i = t; i < ch * T64_W; i += T64_THREADS) {
    const int r = i / T64_W, c = i - r * T64_W;
    double a[4] = {0, 0, 0, 0};
    for (int j = 0; j < K; ++j) {
      const double w = p.w[j];
#pragma unroll
      for (int q = 0; q < 4; ++q) a[q] = fma(w, sc[q][r][c + K - 1 - j], a[q]);
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) hs[q][r][c] = a[q];
  }
  __syncthreads();
  const int iy = iy0 + ty, ix = ix0 + tx;
  if (iy >= p.H || ix >= p.W) return;
  double v[4] = {0, 0, 0, 0};
  for (int j = 0; j < K; ++j) {
    const double w = p.w[j];
#pragma unroll
    for (int q = 0; q < 4; ++q) v[q] = fma(w, hs[q][ty + K - 1 - j][tx], v[q]);
  }
  const long long o = ((long long)pl * p.H + iy) * p.W + ix;
  const double xv = x[o], yv = y[o];
  if (dx) dx[o] = 2.0 * xv * v[0] + yv * v[1] + v[2];
  if (dy) dy[o] = 2.0 * yv * v[0] + xv * v[1] + v[3];
}

// ---------------------------------------------------------------------------
// 2x2 average pool (MS-SSIM pyramid) and its adjoint, float64 planes
// ---------------------------------------------------------------------------
__global__ void pool64_kernel(const double* in, int NC, int H, int W, double* out) {
  const int Ho = H / 2, Wo = W / 2;
  const long long n = (long long)NC * Ho * Wo;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const long long pl = i / ((long long)Ho * Wo);
    const int r = (int)((i / Wo) % Ho), c = (int)(i % Wo);
    const double* s = in + (pl * H + 2 * r) * W + 2 * c;
    out[i] = 0.25 * ((s[0] + s[1]) + (s[W] + s[W + 1]));
  }
}

__global__ void pool64_bwd_kernel(const double* g, int NC, int H, int W, double* dx) {
  const int Ho = H / 2, Wo = W / 2;
  const long long n = (long long)NC * H * W;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const long long pl = i / ((long long)H * W);
    const int r = (int)((i / W) % H), c = (int)(i % W);
    const int pr = r >> 1, pc = c >> 1;
    dx[i] = (pr < Ho && pc < Wo) ? 0.25 * g[(pl * Ho + pr) * Wo + pc] : 0.0;
  }
}

// ---------------------------------------------------------------------------
// GMSD / GMS in float64.  q at map position (i, j) from the pooled plane:
// gx = (P[i..i+2][j] - P[i..i+2][j+2]) / 3 summed over rows, gy likewise
// over columns; g = sqrt(gx^2 + gy^2 + eps); q = (2 g1 g2 + T)/(g1^2 + g2^2 + T)
// (reference.py:288-335).  Per image: mean of q and its population std over
// every plane's map.
// ---------------------------------------------------------------------------
struct Gmsd64Args {
  const char* x;
  const char* y;
  long long sn, sc, sh;
  int N, C, H, W;
  int Cm, P;
  int Hd, Wd, Hout, Wout;
  int down;
  double T, eps;
  double lk0, lk1, lk2, lk3;
  int luma;
  int blocks_pp;  // blocks per plane
  unsigned int* counter;
  double* part;   // [P][blocks_pp][2]
  double* out_mean;
  double* out_std;
  double* map;    // [P][Hout][Wout] q, or null
  // backward
  const double* gmean;  // [N] upstream of the per-image mean
  const double* gstd;   // [N] upstream of the per-image std
  const double* mu;     // [N] forward mean of q
  const double* sd;     // [N] forward std of q
  double* coef;         // [4][P][Hout][Wout]: dL/dgx1, dL/dgy1, dL/dgx2, dL/dgy2
};

template <typename T>
__device__ __forceinline__ double gpx64(const Gmsd64Args& p, const char* base, int pl, int r,
                                        int c) {
  const int n = pl / p.Cm, ch = pl - n * p.Cm;
  const long long o = (long long)n * p.sn + (long long)r * p.sh + c;
  if (p.luma) {
    return fma(p.lk0, ld64<T>(base, o), fma(p.lk1, ld64<T>(base, o + p.sc),
               fma(p.lk2, ld64<T>(base, o + 2 * p.sc), p.lk3)));
  }
  return ld64<T>(base, o + (long long)ch * p.sc);
}

// pooled (or plain) sample
template <typename T>
__device__ __forceinline__ double dpx64(const Gmsd64Args& p, const char* base, int pl, int r,
                                        int c) {
  if (!p.down) return gpx64<T>(p, base, pl, r, c);
  return 0.25 * ((gpx64<T>(p, base, pl, 2 * r, 2 * c) + gpx64<T>(p, base, pl, 2 * r, 2 * c + 1)) +
                 (gpx64<T>(p, base, pl, 2 * r + 1, 2 * c) +
                  gpx64<T>(p, base, pl, 2 * r + 1, 2 * c + 1)));
}

template <typename T>
__device__ __forceinline__ void grad64(const Gmsd64Args& p, const char* base, int pl, int i,
                                       int j, double& gx, double& gy) {
  double v[3][3];
#pragma unroll
  for (int a = 0; a < 3; ++a)
#pragma unroll
    for (int b = 0; b < 3; ++b) v[a][b] = dpx64<T>(p, base, pl, i + a, j + b);
  gx = ((v[0][0] - v[0][2]) + (v[1][0] - v[1][2]) + (v[2][0] - v[2][2])) / 3.0;
  gy = ((v[0][0] + v[0][1] + v[0][2]) - (v[2][0] + v[2][1] + v[2][2])) / 3.0;
}

template <typename T, bool COEF>
__global__ void __launch_bounds__(256) gmsd64_kernel(const Gmsd64Args p) {
  __shared__ double s_red[32];
  __shared__ int s_flag;
  const int pl = blockIdx.y;
  const long long npos = (long long)p.Hout * p.Wout;
  double s = 0.0, s2 = 0.0;
  for (long long k = blockIdx.x * 256LL + threadIdx.x; k < npos; k += 256LL * gridDim.x) {
    const int i = (int)(k / p.Wout), j = (int)(k - (long long)i * p.Wout);
    double gx1, gy1, gx2, gy2;
    grad64<T>(p, p.x, pl, i, j, gx1, gy1);
    grad64<T>(p, p.y, pl, i, j, gx2, gy2);
    const double G1 = gx1 * gx1 + gy1 * gy1 + p.eps, G2 = gx2 * gx2 + gy2 * gy2 + p.eps;
    const double g1 = sqrt(G1), g2 = sqrt(G2);
    const double den = G1 + G2 + p.T;
    const double q = (2.0 * g1 * g2 + p.T) / den;
    const long long o = (long long)pl * npos + k;
    if constexpr (!COEF) {
      const double d = q - 1.0;
      s += d;
      s2 += d * d;
      if (p.map) p.map[o] = q;
    } else {
      // dL/dq: the mean's and the std's upstream gradients over this image's
      // n = planes x positions values
      const int n = pl / p.Cm;
      const double cnt = (double)npos * p.Cm;
      double dq = p.gmean[n] / cnt;
      if (p.sd[n] > 0.0) dq += p.gstd[n] * (q - p.mu[n]) / (cnt * p.sd[n]);
      // dq/dg1 = (2 g2 den - (2 g1 g2 + T) 2 g1) / den^2, and dg1/dgx1 = gx1 / g1
      const double dq1 = (2.0 * g2 - 2.0 * g1 * q) / den;
      const double dq2 = (2.0 * g1 - 2.0 * g2 * q) / den;
      const long long plane = (long long)p.P * npos;
      p.coef[o] = dq * dq1 * gx1 / g1;
      p.coef[o + plane] = dq * dq1 * gy1 / g1;
      p.coef[o + 2 * plane] = dq * dq2 * gx2 / g2;
      p.coef[o + 3 * plane] = dq * dq2 * gy2 / g2;
    }
  }
  if constexpr (!COEF) {
    s = block_sum(s, s_red);
    s2 = block_sum(s2, s_red);
    const long long pidx = ((long long)pl * p.blocks_pp + blockIdx.x) * 2;
    if (threadIdx.x == 0) {
      p.part[pidx] = s;
      p.part[pidx + 1] = s2;
    }
    if (last_block_arrived(p.counter, gridDim.x * gridDim.y, &s_flag)) {
      const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
      const double cnt = (double)npos * p.Cm;
      for (int n = wid; n < p.N; n += 8) {
        double a = 0.0, b = 0.0;
        for (int c = 0; c < p.Cm; ++c)
          for (int i = lane; i < p.blocks_pp; i += 32) {
            a += p.part[((long long)(n * p.Cm + c) * p.blocks_pp + i) * 2];
            b += p.part[((long long)(n * p.Cm + c) * p.blocks_pp + i) * 2 + 1];
          }
        a = warp_sum(a);
        b = warp_sum(b);
        if (lane == 0) {
          const double md = a / cnt, var = b / cnt - md * md;
          if (p.out_mean) p.out_mean[n] = 1.0 + md;
          if (p.out_std) p.out_std[n] = sqrt(var > 0.0 ? var : 0.0);
        }
      }
    }
  }
}

// dL/d(pooled sample) from the coefficient planes through the transposed
// Prewitt/3 filters, then 1/4 to each of its 2x2 inputs (float64 planes,
// contiguous; no luma: the autograd path projects luma with torch first).
__global__ void __launch_bounds__(256) gmsd64_scatter_kernel(const Gmsd64Args p, double* dx,
                                                             double* dy) {
  const long long npos = (long long)p.Hout * p.Wout, plane = (long long)p.P * npos;
  const long long nin = (long long)p.P * p.H * p.W;
  for (long long k = blockIdx.x * 256LL + threadIdx.x; k < nin; k += 256LL * gridDim.x) {
    const int pl = (int)(k / ((long long)p.H * p.W));
    const int r = (int)((k / p.W) % p.H), c = (int)(k % p.W);
    const int pr = p.down ? r >> 1 : r, pc = p.down ? c >> 1 : c;
    double a1 = 0.0, a2 = 0.0;
    if (pr < p.Hd && pc < p.Wd) {
      // pooled (pr, pc) sits at offset (a, b) of the 3x3 window of map
      // position (pr - a, pc - b): gx weight (b == 0) - (b == 2), gy weight
      // (a == 0) - (a == 2), each over 3
      for (int a = 0; a < 3; ++a) {
        const int i = pr - a;
        if (i < 0 || i >= p.Hout) continue;
        for (int b = 0; b < 3; ++b) {
          const int j = pc - b;
          if (j < 0 || j >= p.Wout) continue;
          const double wx = ((b == 0) - (b == 2)) / 3.0, wy = ((a == 0) - (a == 2)) / 3.0;
          const long long o = (long long)pl * npos + (long long)i * p.Wout + j;
          a1 += wx * p.coef[o] + wy * p.coef[o + plane];
          a2 += wx * p.coef[o + 2 * plane] + wy * p.coef[o + 3 * plane];
        }
      }
      if (p.down) {
        a1 *= 0.25;
        a2 *= 0.25;
      }
    }
    if (dx) dx[k] = a1;
    if (dy) dy[k] = a2;
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
template <typename T, bool COEF>
static int launch_ssim64(Ssim64Args& p, cudaStream_t st) {
  dim3 grid(p.tiles_x, p.tiles_y, p.P);
  ssim64_kernel<T, COEF><<<grid, T64_THREADS, 0, st>>>(p);
  FAB_LAUNCH_CHECK();
  return FA_OK;
}

static int ssim64_setup(Ssim64Args& p, const View& x, const View& y, int dtype,
                        const double* luma, const double* taps, int K, double C1, double C2) {
  if (!x.data || !y.data || !taps) return FA_E_ARG;
  if (dtype != FA_F64) return FA_E_DTYPE;
  if (x.n != y.n || x.c != y.c || x.h != y.h || x.w != y.w) return FA_E_SHAPE;
  if (x.sn != y.sn || x.sc != y.sc || x.sh != y.sh) return FA_E_SHAPE;
  if (K < 1 || K > MAXK) return FA_E_WINDOW;
  if (luma && x.c != 3) return FA_E_SHAPE;
  p = Ssim64Args{};
  p.x = static_cast<const char*>(x.data);
  p.y = static_cast<const char*>(y.data);
  p.sn = x.sn; p.sc = x.sc; p.sh = x.sh;
  p.N = x.n; p.C = x.c; p.H = x.h; p.W = x.w;
  p.Cm = luma ? 1 : x.c;
  p.P = p.N * p.Cm;
  p.Hout = x.h - K + 1; p.Wout = x.w - K + 1;
  if (p.Hout <= 0 || p.Wout <= 0) return FA_E_SHAPE;
  if (p.P > 65535) return FA_E_SHAPE;
  p.K = K;
  for (int j = 0; j < K; ++j) p.w[j] = taps[j];
  p.C1 = C1; p.C2 = C2;
  if (luma) {
    p.luma = 1;
    p.lk0 = luma[0]; p.lk1 = luma[1]; p.lk2 = luma[2]; p.lk3 = luma[3];
  }
  p.tiles_x = (p.Wout + T64_W - 1) / T64_W;
  p.tiles_y = (p.Hout + T64_H - 1) / T64_H;
  return FA_OK;
}

size_t ssim64_ws_bytes(int planes, int h, int w, int K) {
  const long long tx = (w - K + 1 + T64_W - 1) / T64_W, ty = (h - K + 1 + T64_H - 1) / T64_H;
  if (tx <= 0 || ty <= 0) return FAB_COUNTER_BYTES;
  return FAB_COUNTER_BYTES + 2 * sizeof(double) * (size_t)planes * tx * ty;
}

int ssim64_fwd_impl(const View& x, const View& y, int dtype, const double* luma,
                    const double* taps, int K, double C1, double C2, void* ws, size_t ws_bytes,
                    double* map, double* out_plane_s, double* out_plane_cs,
                    double* out_per_image, double* out_total, cudaStream_t st) {
  Ssim64Args p;
  if (const int rc = ssim64_setup(p, x, y, dtype, luma, taps, K, C1, C2)) return rc;
  if (!ws) return FA_E_ARG;
  const size_t nb = (size_t)p.P * p.tiles_x * p.tiles_y;
  if (ws_bytes < FAB_COUNTER_BYTES + 2 * sizeof(double) * nb) return FA_E_ARG;
  p.counter = static_cast<unsigned int*>(ws);
  p.part_s = reinterpret_cast<double*>(static_cast<char*>(ws) + FAB_COUNTER_BYTES);
  p.part_cs = out_plane_cs ? p.part_s + nb : nullptr;
  p.map = map;
  p.out_plane_s = out_plane_s; p.out_plane_cs = out_plane_cs;
  p.out_per_image = out_per_image; p.out_total = out_total;
  return launch_ssim64<double, false>(p, st);
}

int ssim64_bwd_impl(const double* x, const double* y, int N, int C, int H, int W,
                    const double* taps, int K, double C1, double C2, const double* dmap,
                    const double* gscalar, const double* gs, const double* gcs, double* coef,
                    double* dx, double* dy, cudaStream_t st) {
  const int forms = (dmap ? 1 : 0) + (gscalar ? 1 : 0) + ((gs || gcs) ? 1 : 0);
  if (forms != 1 || !coef || (!dx && !dy)) return FA_E_ARG;
  if ((gs != nullptr) != (gcs != nullptr)) return FA_E_ARG;
  if (N <= 0 || C <= 0 || H <= 0 || W <= 0) return FA_E_SHAPE;
  View vx{x, N, C, H, W, (long long)C * H * W, (long long)H * W, W};
  View vy{y, N, C, H, W, (long long)C * H * W, (long long)H * W, W};
  Ssim64Args p;
  if (const int rc = ssim64_setup(p, vx, vy, FA_F64, nullptr, taps, K, C1, C2)) return rc;
  p.gmode = dmap ? 0 : (gscalar ? 1 : 2);
  p.dmap = dmap; p.gscalar = gscalar; p.gs = gs; p.gcs = gcs;
  const double npix = (double)p.Hout * p.Wout;
  p.grad_norm = gscalar ? 1.0 / (npix * p.P) : (gs ? 1.0 / npix : 1.0);
  p.coef = coef;
  if (const int rc = launch_ssim64<double, true>(p, st)) return rc;
  dim3 grid((W + T64_W - 1) / T64_W, (H + T64_H - 1) / T64_H, p.P);
  ssim64_scatter_kernel<<<grid, T64_THREADS, 0, st>>>(p, x, y, dx, dy);
  FAB_LAUNCH_CHECK();
  return FA_OK;
}

int pool64_impl(const double* in, int NC, int H, int W, double* out, int device,
                cudaStream_t st) {
  if (!in || !out) return FA_E_ARG;
  if (NC <= 0 || H < 2 || W < 2) return FA_E_SHAPE;
  const long long n = (long long)NC * (H / 2) * (W / 2);
  const long long cap = (long long)sm_count(device) * 8;
  const unsigned blocks = (unsigned)std::min<long long>((n + 255) / 256, cap);
  pool64_kernel<<<blocks, 256, 0, st>>>(in, NC, H, W, out);
  FAB_LAUNCH_CHECK();
  return FA_OK;
}

int pool64_bwd_impl(const double* g, int NC, int H, int W, double* dx, int device,
                    cudaStream_t st) {
  if (!g || !dx) return FA_E_ARG;
  if (NC <= 0 || H < 2 || W < 2) return FA_E_SHAPE;
  const long long n = (long long)NC * H * W;
  const long long cap = (long long)sm_count(device) * 8;
  const unsigned blocks = (unsigned)std::min<long long>((n + 255) / 256, cap);
  pool64_bwd_kernel<<<blocks, 256, 0, st>>>(g, NC, H, W, dx);
  FAB_LAUNCH_CHECK();
  return FA_OK;
}

static int gmsd64_setup(Gmsd64Args& p, const View& x, const View& y, int dtype,
                        const double* luma, double T, double eps, int down, int device) {
  if (!x.data || !y.data) return FA_E_ARG;
  if (dtype != FA_F64) return FA_E_DTYPE;
  if (x.n != y.n || x.c != y.c || x.h != y.h || x.w != y.w) return FA_E_SHAPE;
  if (x.sn != y.sn || x.sc != y.sc || x.sh != y.sh) return FA_E_SHAPE;
  if (luma && x.c != 3) return FA_E_SHAPE;
  p = Gmsd64Args{};
  p.x = static_cast<const char*>(x.data);
  p.y = static_cast<const char*>(y.data);
  p.sn = x.sn; p.sc = x.sc; p.sh = x.sh;
  p.N = x.n; p.C = x.c; p.H = x.h; p.W = x.w;
  p.Cm = luma ? 1 : x.c;
  p.P = p.N * p.Cm;
  p.down = down ? 1 : 0;
  p.Hd = down ? x.h / 2 : x.h;
  p.Wd = down ? x.w / 2 : x.w;
  p.Hout = p.Hd - 2; p.Wout = p.Wd - 2;
  if (p.Hout <= 0 || p.Wout <= 0) return FA_E_SHAPE;
  if (p.P > 65535) return FA_E_SHAPE;
  p.T = T; p.eps = eps;
  if (luma) {
    p.luma = 1;
    p.lk0 = luma[0]; p.lk1 = luma[1]; p.lk2 = luma[2]; p.lk3 = luma[3];
  }
  const long long npos = (long long)p.Hout * p.Wout;
  long long bpp = (sm_count(device) * 8LL + p.P - 1) / p.P;
  bpp = std::max(1LL, std::min(bpp, (npos + 255) / 256));
  p.blocks_pp = (int)bpp;
  return FA_OK;
}

size_t gmsd64_ws_bytes(int planes, int h, int w, int down, int device) {
  const int hd = down ? h / 2 : h, wd = down ? w / 2 : w;
  const long long npos = (long long)(hd - 2) * (wd - 2);
  if (npos <= 0) return FAB_COUNTER_BYTES;
  long long bpp = (sm_count(device) * 8LL + planes - 1) / planes;
  bpp = std::max(1LL, std::min(bpp, (npos + 255) / 256));
  return FAB_COUNTER_BYTES + 2 * sizeof(double) * (size_t)planes * bpp;
}

int gmsd64_impl(const View& x, const View& y, int dtype, const double* luma, double T,
                double eps, int down, void* ws, size_t ws_bytes, double* map,
                double* out_mean, double* out_std, int device, cudaStream_t st) {
  Gmsd64Args p;
  if (const int rc = gmsd64_setup(p, x, y, dtype, luma, T, eps, down, device)) return rc;
  if (!ws || ws_bytes < FAB_COUNTER_BYTES + 2 * sizeof(double) * (size_t)p.P * p.blocks_pp)
    return FA_E_ARG;
  p.counter = static_cast<unsigned int*>(ws);
  p.part = reinterpret_cast<double*>(static_cast<char*>(ws) + FAB_COUNTER_BYTES);
  p.map = map;
  p.out_mean = out_mean; p.out_std = out_std;
  dim3 grid(p.blocks_pp, p.P);
  gmsd64_kernel<double, false><<<grid, 256, 0, st>>>(p);
  FAB_LAUNCH_CHECK();
  return FA_OK;
}

int gmsd64_bwd_impl(const double* x, const double* y, int N, int C, int H, int W, int down,
                    double T, double eps, const double* gm, const double* gsd, const double* mu,
                    const double* sd, double* coef, double* dx, double* dy, int device,
                    cudaStream_t st) {
  if (!gm || !gsd || !mu || !sd || !coef || (!dx && !dy)) return FA_E_ARG;
  if (N <= 0 || C <= 0 || H <= 0 || W <= 0) return FA_E_SHAPE;
  View vx{x, N, C, H, W, (long long)C * H * W, (long long)H * W, W};
  View vy{y, N, C, H, W, (long long)C * H * W, (long long)H * W, W};
  Gmsd64Args p;
  if (const int rc = gmsd64_setup(p, vx, vy, FA_F64, nullptr, T, eps, down, device)) return rc;
  p.gmean = gm; p.gstd = gsd; p.mu = mu; p.sd = sd; p.coef = coef;
  dim3 grid(p.blocks_pp, p.P);
  gmsd64_kernel<double, true><<<grid, 256, 0, st>>>(p);
  FAB_LAUNCH_CHECK();
  const long long nin = (long long)p.P * H * W;
  const unsigned blocks = (unsigned)std::min<long long>((nin + 255) / 256, sm_count(device) * 8LL);
  gmsd64_scatter_kernel<<<blocks, 256, 0, st>>>(p, dx, dy);
  FAB_LAUNCH_CHECK();
  return FA_OK;
}

}  // namespace fab
