// GMSD / GMS on sm_100a.
//
// Semantics (reference: frame_analytics/reference.py:284-335 and the fused
// kernel fa_cuda.cu:926-1026):
//   optional 2x2 non-overlapping mean (odd trailing row/column dropped),
//   valid Prewitt/3 pair, g = sqrt(gx^2 + gy^2 + eps),
//   q = (2 g1 g2 + T) / (g1^2 + g2^2 + T),
//   per image: mean and population std of q pooled over all channels' maps.
//
// Design (B200, near the HBM ridge): a block owns a strip of 512 pooled
// columns and streams down a chunk of rows; every input byte is read once.
// Each thread pools 4 adjacent columns per row (one 8-byte load per input row
// for uint8).  Pooled rows live in a shared-memory ring that carries the two
// halo rows between iterations.  The map is accumulated as d = q - 1 =
// -(g1 - g2)^2 / (g1^2 + g2^2 + T), which is exact to rounding where q is
// close to 1, so sum(d) and sum(d^2) give the variance without cancellation.
// Last-block finalisation keeps the whole metric to one launch.
#include "common.cuh"

namespace fab {

constexpr int GM_T = 128;             // threads
constexpr int GM_CPT = 4;             // pooled columns per thread
constexpr int GM_DW = GM_T * GM_CPT;  // pooled columns staged per strip
constexpr int GM_OW = GM_DW - 2;      // output columns per strip
constexpr int GM_R = 8;               // output rows per iteration
constexpr int GM_RING = GM_R + 2;

struct GmsdArgs {
  const char* x;
  const char* y;
  long long sn, sc, sh;
  int N, C, H, W;
  int P, Cm;
  int Hd, Wd;      // pooled (or input) size
  int Hout, Wout;  // map size
  float T, eps;
  float lk0, lk1, lk2, lk3;
  int strips, chunks, RH;
  unsigned int* counter;
  double* part;    // [P][bpp][2]
  double* out_mean;
  double* out_std;
  float* map;      // optional [P][Hout][Wout] GMS map
};

template <typename T, bool LUMA>
__device__ __forceinline__ float gm_px(const GmsdArgs& p, const T* X, long long o) {
  if constexpr (LUMA) {
    return fmaf(p.lk0, Ld<T>::f(ldro(X + o)),
                fmaf(p.lk1, Ld<T>::f(ldro(X + o + p.sc)),
                     fmaf(p.lk2, Ld<T>::f(ldro(X + o + 2 * p.sc)), p.lk3)));
  } else {
    return Ld<T>::f(ldro(X + o));
  }
}

// Pooled values of 4 adjacent pooled columns (dc .. dc+3) of pooled row dr.
template <typename T, bool DOWN, bool LUMA>
__device__ __forceinline__ void gm_load4(const GmsdArgs& p, const T* X, long long base,
                                         int dr, int dc, float (&v)[GM_CPT]) {
  if constexpr (DOWN && !LUMA && sizeof(T) == 1) {
    const long long o0 = base + (long long)(2 * dr) * p.sh + 2 * dc;
    const unsigned char* b0 = reinterpret_cast<const unsigned char*>(X) + o0;
    const unsigned char* b1 = b0 + p.sh;
    if (dc + GM_CPT <= p.Wd && ((reinterpret_cast<uintptr_t>(b0) | reinterpret_cast<uintptr_t>(b1)) & 7u) == 0) {
      const uint2 u0 = __ldg(reinterpret_cast<const uint2*>(b0));
      const uint2 u1 = __ldg(reinterpret_cast<const uint2*>(b1));
      const unsigned a[2] = {u0.x, u0.y};
      const unsigned b[2] = {u1.x, u1.y};
#pragma unroll
      for (int i = 0; i < GM_CPT; ++i) {
        const unsigned wa = a[i >> 1] >> ((i & 1) * 16);
        const unsigned wb = b[i >> 1] >> ((i & 1) * 16);
        const int s = (int)(wa & 0xff) + (int)((wa >> 8) & 0xff) + (int)(wb & 0xff) +
                      (int)((wb >> 8) & 0xff);
        v[i] = 0.25f * (float)s;
      }
      return;
    }
  }
#pragma unroll
  for (int i = 0; i < GM_CPT; ++i) {
    const int c = dc + i;
    float r = 0.f;
    if (c < p.Wd) {
      if constexpr (DOWN) {
        const long long o = base + (long long)(2 * dr) * p.sh + 2 * c;
        r = 0.25f * (gm_px<T, LUMA>(p, X, o) + gm_px<T, LUMA>(p, X, o + 1) +
                     gm_px<T, LUMA>(p, X, o + p.sh) + gm_px<T, LUMA>(p, X, o + p.sh + 1));
      } else {
        r = gm_px<T, LUMA>(p, X, base + (long long)dr * p.sh + c);
      }
    }
    v[i] = r;
  }
}

__device__ void gmsd_finalize(const GmsdArgs& p, int bpp) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int nw = blockDim.x >> 5;
  const double npix = (double)p.Hout * p.Wout * p.Cm;
  for (int n = wid; n < p.N; n += nw) {
    double s = 0.0, s2 = 0.0;
    for (int c = 0; c < p.Cm; ++c) {
      const double* row = p.part + (long long)(n * p.Cm + c) * bpp * 2;
      for (int i = lane; i < bpp; i += 32) {
        s += row[2 * i];
        s2 += row[2 * i + 1];
      }
    }
    s = warp_sum(s);
    s2 = warp_sum(s2);
    if (lane == 0) {
      const double md = s / npix;
      const double var = s2 / npix - md * md;
      if (p.out_mean) p.out_mean[n] = 1.0 + md;
      if (p.out_std) p.out_std[n] = sqrt(var > 0.0 ? var : 0.0);
    }
  }
}

template <typename T, bool DOWN, bool LUMA>
__global__ void __launch_bounds__(GM_T) gmsd_kernel(GmsdArgs p) {
  __shared__ float sx[GM_RING][GM_DW + 4];
  __shared__ float sy[GM_RING][GM_DW + 4];
  __shared__ double s_red[32];
  __shared__ int s_flag;

  const int t = threadIdx.x;
  const int plane = blockIdx.z;
  const int pn = plane / p.Cm, pc = plane - pn * p.Cm;
  const long long base = (long long)pn * p.sn + (long long)pc * p.sc;
  const T* X = reinterpret_cast<const T*>(p.x);
  const T* Y = reinterpret_cast<const T*>(p.y);
  const int dc0 = blockIdx.x * GM_OW;  // first pooled column of the strip
  const int r0 = blockIdx.y * p.RH;    // first output row of the chunk
  const int rows = min(p.RH, p.Hout - r0);
  const int dc = dc0 + t * GM_CPT;

  // first two pooled rows of the chunk
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    float a[GM_CPT], b[GM_CPT];
    const int dr = r0 + k;
    gm_load4<T, DOWN, LUMA>(p, X, base, dr, dc, a);
    gm_load4<T, DOWN, LUMA>(p, Y, base, dr, dc, b);
#pragma unroll
    for (int i = 0; i < GM_CPT; ++i) {
      sx[k][t * GM_CPT + i] = a[i];
      sy[k][t * GM_CPT + i] = b[i];
    }
  }
  double acc = 0.0, acc2 = 0.0;
  for (int rb = 0; rb < rows; rb += GM_R) {
    const int nr = min(GM_R, rows - rb);
    // pooled rows rb+2 .. rb+nr+1 into ring rows 2 .. nr+1
    for (int k = 0; k < nr; ++k) {
      float a[GM_CPT], b[GM_CPT];
      const int dr = r0 + rb + 2 + k;
      gm_load4<T, DOWN, LUMA>(p, X, base, dr, dc, a);
      gm_load4<T, DOWN, LUMA>(p, Y, base, dr, dc, b);
#pragma unroll
      for (int i = 0; i < GM_CPT; ++i) {
        sx[2 + k][t * GM_CPT + i] = a[i];
        sy[2 + k][t * GM_CPT + i] = b[i];
      }
    }
    __syncthreads();
    float fs = 0.f, fs2 = 0.f;
    constexpr float THIRD = 1.0f / 3.0f;
    for (int k = 0; k < nr; ++k) {
#pragma unroll
      for (int i = 0; i < GM_CPT; ++i) {
        const int c = t * GM_CPT + i;
        if (c < GM_OW && dc0 + c < p.Wout) {
          float g[2];
#pragma unroll
          for (int which = 0; which < 2; ++which) {
            const float(*s)[GM_DW + 4] = which ? sy : sx;
            const float gx = ((s[k][c] - s[k][c + 2]) + (s[k + 1][c] - s[k + 1][c + 2]) +
                              (s[k + 2][c] - s[k + 2][c + 2])) * THIRD;
            const float gy = ((s[k][c] - s[k + 2][c]) + (s[k][c + 1] - s[k + 2][c + 1]) +
                              (s[k][c + 2] - s[k + 2][c + 2])) * THIRD;
            g[which] = sqrtf(fmaf(gx, gx, fmaf(gy, gy, p.eps)));
          }
          const float dg = g[0] - g[1];
          const float d = -(dg * dg) / fmaf(g[0], g[0], fmaf(g[1], g[1], p.T));
          fs += d;
          fs2 = fmaf(d, d, fs2);
          if (p.map)
            p.map[((long long)plane * p.Hout + (r0 + rb + k)) * p.Wout + dc0 + c] = 1.0f + d;
        }
      }
    }
    acc += (double)fs;
    acc2 += (double)fs2;
    __syncthreads();
    // carry the last two pooled rows to the top of the ring
    for (int i = t; i < GM_DW; i += GM_T) {
      sx[0][i] = sx[nr][i];
      sx[1][i] = sx[nr + 1][i];
      sy[0][i] = sy[nr][i];
      sy[1][i] = sy[nr + 1][i];
    }
    __syncthreads();
  }
  const int bpp = p.strips * p.chunks;
  const long long pidx = ((long long)plane * bpp + blockIdx.y * p.strips + blockIdx.x) * 2;
  acc = block_sum(acc, s_red);
  if (t == 0) p.part[pidx] = acc;
  acc2 = block_sum(acc2, s_red);
  if (t == 0) p.part[pidx + 1] = acc2;
  if (last_block_arrived(p.counter, gridDim.x * gridDim.y * gridDim.z, &s_flag))
    gmsd_finalize(p, bpp);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
struct GmPlan {
  int strips, chunks, RH;
};

static GmPlan gm_plan(int Hout, int Wout, int planes, int device) {
  GmPlan g;
  g.strips = (Wout + GM_OW - 1) / GM_OW;
  const int sms = sm_count(device);
  // ~12 resident blocks per SM, a few waves
  long long want = (24LL * sms + (long long)g.strips * planes - 1) / ((long long)g.strips * planes);
  if (want < 1) want = 1;
  long long maxc = (Hout + GM_R - 1) / GM_R;
  if (want > maxc) want = maxc;
  g.RH = (int)((Hout + want - 1) / want);
  g.RH = ((g.RH + GM_R - 1) / GM_R) * GM_R;
  g.chunks = (Hout + g.RH - 1) / g.RH;
  return g;
}

static bool gm_dims(int h, int w, int down, int* Hd, int* Wd, int* Ho, int* Wo) {
  *Hd = down ? h / 2 : h;
  *Wd = down ? w / 2 : w;
  *Ho = *Hd - 2;
  *Wo = *Wd - 2;
  return *Ho > 0 && *Wo > 0;
}

size_t gmsd_ws_bytes(int planes, int h, int w, int down, int device) {
  int Hd, Wd, Ho, Wo;
  if (!gm_dims(h, w, down, &Hd, &Wd, &Ho, &Wo)) return FAB_COUNTER_BYTES;
  const GmPlan g = gm_plan(Ho, Wo, planes, device);
  return FAB_COUNTER_BYTES + 2 * sizeof(double) * (size_t)planes * g.strips * g.chunks;
}

template <typename T, bool DOWN, bool LUMA>
static int gm_launch(GmsdArgs& p, cudaStream_t st) {
  dim3 grid(p.strips, p.chunks, p.P);
  gmsd_kernel<T, DOWN, LUMA><<<grid, GM_T, 0, st>>>(p);
  FAB_LAUNCH_CHECK();
  return FA_OK;
}

template <typename T>
static int gm_disp(GmsdArgs& p, int down, bool luma, cudaStream_t st) {
  if (down) return luma ? gm_launch<T, true, true>(p, st) : gm_launch<T, true, false>(p, st);
  return luma ? gm_launch<T, false, true>(p, st) : gm_launch<T, false, false>(p, st);
}

int gmsd_impl(const View& x, const View& y, int dtype, const double* luma, double T,
              double eps, int down, void* ws, size_t ws_bytes, float* map_out,
              double* out_mean, double* out_std, int device, cudaStream_t st) {
  if (!x.data || !y.data || !ws) return FA_E_ARG;
  if (x.n <= 0 || x.c <= 0 || x.h <= 0 || x.w <= 0) return FA_E_SHAPE;
  if (x.n != y.n || x.c != y.c || x.h != y.h || x.w != y.w) return FA_E_SHAPE;
  if (x.sn != y.sn || x.sc != y.sc || x.sh != y.sh) return FA_E_SHAPE;
  if (luma && x.c != 3) return FA_E_SHAPE;
  GmsdArgs p{};
  if (!gm_dims(x.h, x.w, down, &p.Hd, &p.Wd, &p.Hout, &p.Wout)) return FA_E_SHAPE;
  p.x = static_cast<const char*>(x.data);
  p.y = static_cast<const char*>(y.data);
  p.sn = x.sn; p.sc = x.sc; p.sh = x.sh;
  p.N = x.n; p.C = x.c; p.H = x.h; p.W = x.w;
  p.Cm = luma ? 1 : x.c;
  p.P = p.N * p.Cm;
  if (p.P > 65535) return FA_E_SHAPE;
  p.T = (float)T; p.eps = (float)eps;
  if (luma) {
    p.lk0 = (float)luma[0]; p.lk1 = (float)luma[1]; p.lk2 = (float)luma[2]; p.lk3 = (float)luma[3];
  }
  const GmPlan g = gm_plan(p.Hout, p.Wout, p.P, device);
  p.strips = g.strips; p.chunks = g.chunks; p.RH = g.RH;
  const size_t need = FAB_COUNTER_BYTES + 2 * sizeof(double) * (size_t)p.P * g.strips * g.chunks;
  if (ws_bytes < need) return FA_E_ARG;
  p.counter = static_cast<unsigned int*>(ws);
  p.part = reinterpret_cast<double*>(static_cast<char*>(ws) + FAB_COUNTER_BYTES);
  p.out_mean = out_mean; p.out_std = out_std;
  p.map = map_out;
  switch (dtype) {
    case FA_U8: return gm_disp<unsigned char>(p, down, luma != nullptr, st);
    case FA_F16: return gm_disp<f16_t>(p, down, luma != nullptr, st);
    case FA_BF16: return gm_disp<bf16_t>(p, down, luma != nullptr, st);
    case FA_F32: return gm_disp<float>(p, down, luma != nullptr, st);
    case FA_F64: return gm_disp<double>(p, down, luma != nullptr, st);
    default: return FA_E_DTYPE;
  }
}

}  // namespace fab
