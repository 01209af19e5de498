// 2x2 mean pooling between the scales of the MS-SSIM pyramid, and the f x f
// box downsample of SSIM's MATLAB mode.
//
// The reference pools with torch (`F.avg_pool2d(x.to(float32), 2)`,
// functional.py:717-725, used at :885 and :930), which for uint8 input first materialises a
// full-resolution float copy.  This kernel reads the input once in its own
// dtype and layout (strided views, optional luma projection) and writes the
// pooled float32 plane: out = (a + b + c + d) / 4 over non-overlapping 2x2
// blocks, an odd trailing row/column dropped (reference.py:231-241, `_avg_pool2`).
// Its backward spreads a quarter of each pooled gradient over the 2x2 block.
// Both are bandwidth-bound elementwise kernels: each thread produces two
// adjacent outputs.
#include "common.cuh"

namespace fab {

struct PoolArgs {
  const char* x;
  long long sn, sc, sh;
  int N, C, H, W, Cm, Hp, Wp;
  float k0, k1, k2, k3;
  float* out;
};

template <typename T, bool LUMA>
__device__ __forceinline__ float pool_px(const PoolArgs& p, const T* X, long long o) {
  if constexpr (LUMA) {
    return fmaf(p.k0, Ld<T>::f(ldro(X + o)),
                fmaf(p.k1, Ld<T>::f(ldro(X + o + p.sc)), fmaf(p.k2, Ld<T>::f(ldro(X + o + 2 * p.sc)), p.k3)));
  } else {
    return Ld<T>::f(ldro(X + o));
  }
}

template <typename T, bool LUMA>
__global__ void __launch_bounds__(256) pool2_kernel(PoolArgs p) {
  const T* X = reinterpret_cast<const T*>(p.x);
  const int wp2 = (p.Wp + 1) / 2;  // output pairs per row
  const long long total = (long long)p.N * p.Cm * p.Hp * wp2;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int j2 = (int)(i % wp2);
    long long r = i / wp2;
    const int hp = (int)(r % p.Hp);
    r /= p.Hp;
    const int c = (int)(r % p.Cm);
    const int n = (int)(r / p.Cm);
    const long long base = (long long)n * p.sn + (long long)c * p.sc + (long long)(2 * hp) * p.sh;
    float* o = p.out + (((long long)n * p.Cm + c) * p.Hp + hp) * p.Wp;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int j = 2 * j2 + k;
      if (j < p.Wp) {
        const long long a = base + 2 * j;
        const float s = pool_px<T, LUMA>(p, X, a) + pool_px<T, LUMA>(p, X, a + 1) +
                        pool_px<T, LUMA>(p, X, a + p.sh) + pool_px<T, LUMA>(p, X, a + p.sh + 1);
        o[j] = 0.25f * s;
      }
    }
  }
}

// Vector path (no luma; 16-byte aligned base and strides; W a multiple of
// V = 16 / sizeof(T)): one thread reads a 16-byte chunk of each of the two
// rows and writes V/2 pooled values, float4 stores when the output rows are
// 16-byte aligned.  The sum order (a + b + c + d, row-major in the block) is
// that of the scalar path.
template <typename T>
struct Vec16 {
  static constexpr int V = 16 / (int)sizeof(T);
  __device__ static __forceinline__ void load(const T* p, float (&v)[V]) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
    const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int i = 0; i < V; ++i) v[i] = Ld<T>::f(e[i]);
  }
};

template <typename T, bool VST>
__global__ void __launch_bounds__(256) pool2_vec_kernel(PoolArgs p) {
  constexpr int V = Vec16<T>::V;
  const T* X = reinterpret_cast<const T*>(p.x);
  const int nch = p.W / V;  // chunks per row
  const long long total = (long long)p.N * p.C * p.Hp * nch;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int ch = (int)(i % nch);
    long long r = i / nch;
    const int hp = (int)(r % p.Hp);
    r /= p.Hp;
    const int c = (int)(r % p.C);
    const int n = (int)(r / p.C);
    const T* a = X + (long long)n * p.sn + (long long)c * p.sc + (long long)(2 * hp) * p.sh +
                 (long long)ch * V;
    float u[V], w[V];
    Vec16<T>::load(a, u);
    Vec16<T>::load(a + p.sh, w);
    float o[V / 2];
#pragma unroll
    for (int k = 0; k < V / 2; ++k) o[k] = 0.25f * (u[2 * k] + u[2 * k + 1] + w[2 * k] + w[2 * k + 1]);
    float* out = p.out + (((long long)n * p.C + c) * p.Hp + hp) * p.Wp + (long long)ch * (V / 2);
    if constexpr (VST && V / 2 >= 4) {
#pragma unroll
      for (int k = 0; k < V / 2; k += 4)
        *reinterpret_cast<float4*>(out + k) = make_float4(o[k], o[k + 1], o[k + 2], o[k + 3]);
    } else if constexpr (VST && V / 2 == 2) {
      *reinterpret_cast<float2*>(out) = make_float2(o[0], o[1]);
    } else {
#pragma unroll
      for (int k = 0; k < V / 2; ++k) out[k] = o[k];
    }
  }
}

__global__ void __launch_bounds__(256) pool2_bwd_kernel(const float* __restrict__ g, int NC, int H,
                                                         int W, int Hp, int Wp,
                                                         float* __restrict__ dx) {
  const long long total = (long long)NC * H * W;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int w = (int)(i % W);
    const long long r = i / W;
    const int h = (int)(r % H);
    const long long pl = r / H;
    const int hp = h >> 1, wp = w >> 1;
    dx[i] = (hp < Hp && wp < Wp) ? 0.25f * __ldg(g + (pl * Hp + hp) * Wp + wp) : 0.f;
  }
}

// MATLAB ssim.m's automatic downsample for large images (the reference's
// _matlab_downsample, functional.py:575-586): an f x f box mean over the
// image with replicated borders (pad f/2 on each side), sampled every f-th
// row and column:
//   out[i, j] = 1/f^2 * sum_{a,b < f} x[clamp(f i + a - f/2), clamp(f j + b - f/2)]
// Output (ceil((H + 2 pad - f + 1) / f), same for W), float32; luma projects
// RGB first.  One thread per output, the box read straight from the input
// (each input sample is read by one output, or a few on the replicated edge).
template <typename T, bool LUMA>
__global__ void __launch_bounds__(256) box_down_kernel(PoolArgs p, int f, int pad, float wgt) {
  const T* X = reinterpret_cast<const T*>(p.x);
  const long long total = (long long)p.N * p.Cm * p.Hp * p.Wp;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int j = (int)(i % p.Wp);
    long long r = i / p.Wp;
    const int oi = (int)(r % p.Hp);
    r /= p.Hp;
    const int c = (int)(r % p.Cm);
    const int n = (int)(r / p.Cm);
    const long long base = (long long)n * p.sn + (long long)c * p.sc;
    float acc = 0.f;
    for (int a = 0; a < f; ++a) {
      const int gr = min(max(f * oi + a - pad, 0), p.H - 1);
      const long long rb = base + (long long)gr * p.sh;
      for (int b = 0; b < f; ++b) {
        const int gc = min(max(f * j + b - pad, 0), p.W - 1);
        acc = fmaf(wgt, pool_px<T, LUMA>(p, X, rb + gc), acc);
      }
    }
    p.out[i] = acc;
  }
}

// Adjoint of box_down_kernel (no luma).  The boxes tile the padded image
// with stride f, so padded row pr belongs to box (pr + pad) / f when that box
// is sampled.  Input row r stands for padded row r, plus rows -pad..-1 when
// r = 0 and rows H..H+pad-1 when r = H-1 (the replicated border); columns
// likewise.  dx[r, c] = wgt * sum over those rows and columns of g[box].
__device__ __forceinline__ int box_rows(int r, int n, int f, int pad, int nb, int (&idx)[2],
                                        int (&cnt)[2]) {
  // boxes reached from input index r and how many padded copies reach each
  int lo = r, hi = r;
  if (r == 0) lo = -pad;
  if (r == n - 1) hi = n - 1 + pad;
  int m = 0;
  for (int pr = lo; pr <= hi; ++pr) {
    const int b = (pr + pad) / f;
    if (pr + pad < 0 || b >= nb) continue;
    if (m > 0 && idx[m - 1] == b) {
      ++cnt[m - 1];
    } else if (m < 2) {
      idx[m] = b;
      cnt[m] = 1;
      ++m;
    }
  }
  return m;
}

__global__ void __launch_bounds__(256) box_down_bwd_kernel(const float* __restrict__ g, int NC,
                                                            int H, int W, int f, int pad,
                                                            int Hp, int Wp, float wgt,
                                                            float* __restrict__ dx) {
  const long long total = (long long)NC * H * W;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(i % W);
    const long long rr = i / W;
    const int r = (int)(rr % H);
    const long long pl = rr / H;
    int ri[2], rc[2], ci[2], cc[2];
    const int nr = box_rows(r, H, f, pad, Hp, ri, rc);
    const int nc = box_rows(c, W, f, pad, Wp, ci, cc);
    float acc = 0.f;
    for (int a = 0; a < nr; ++a)
      for (int b = 0; b < nc; ++b)
        acc += (float)(rc[a] * cc[b]) * __ldg(g + (pl * Hp + ri[a]) * Wp + ci[b]);
    dx[i] = wgt * acc;
  }
}

static unsigned grid_for(long long work, int device) {
  long long b = (work + 255) / 256;
  const long long cap = (long long)sm_count(device) * 16;
  return (unsigned)(b < 1 ? 1 : (b > cap ? cap : b));
}

template <typename T>
static int pool_launch(const PoolArgs& p, bool luma, int device, cudaStream_t st) {
  constexpr int V = Vec16<T>::V;
  const bool vec = !luma && V >= 2 && p.W % V == 0 &&
                   ((reinterpret_cast<uintptr_t>(p.x) |
                     (uintptr_t)(p.sh * (long long)sizeof(T)) |
                     (uintptr_t)(p.sc * (long long)sizeof(T)) |
                     (uintptr_t)(p.sn * (long long)sizeof(T))) & 15u) == 0;
  if (vec) {
    const long long work = (long long)p.N * p.C * p.Hp * (p.W / V);
    const bool vst = (reinterpret_cast<uintptr_t>(p.out) & 15u) == 0 && (p.Wp * 4) % 16 == 0 &&
                     V / 2 >= 2;
    if (vst) pool2_vec_kernel<T, true><<<grid_for(work, device), 256, 0, st>>>(p);
    else pool2_vec_kernel<T, false><<<grid_for(work, device), 256, 0, st>>>(p);
    FAB_LAUNCH_CHECK();
    return FA_OK;
  }
  const long long work = (long long)p.N * p.Cm * p.Hp * ((p.Wp + 1) / 2);
  if (luma) pool2_kernel<T, true><<<grid_for(work, device), 256, 0, st>>>(p);
  else pool2_kernel<T, false><<<grid_for(work, device), 256, 0, st>>>(p);
  FAB_LAUNCH_CHECK();
  return FA_OK;
}

int pool2_impl(const View& x, int dtype, const double* luma, float* out, int device,
               cudaStream_t st) {
  if (!x.data || !out) return FA_E_ARG;
  if (x.n <= 0 || x.c <= 0 || x.h < 2 || x.w < 2) return FA_E_SHAPE;
  if (luma && x.c != 3) return FA_E_SHAPE;
  PoolArgs p{};
  p.x = static_cast<const char*>(x.data);
  p.sn = x.sn; p.sc = x.sc; p.sh = x.sh;
  p.N = x.n; p.C = x.c; p.H = x.h; p.W = x.w;
  p.Cm = luma ? 1 : x.c;
  p.Hp = x.h / 2; p.Wp = x.w / 2;
  if (luma) {
    p.k0 = (float)luma[0]; p.k1 = (float)luma[1]; p.k2 = (float)luma[2]; p.k3 = (float)luma[3];
  }
  p.out = out;
  switch (dtype) {
    case FA_U8: return pool_launch<unsigned char>(p, luma != nullptr, device, st);
    case FA_F16: return pool_launch<f16_t>(p, luma != nullptr, device, st);
    case FA_BF16: return pool_launch<bf16_t>(p, luma != nullptr, device, st);
    case FA_F32: return pool_launch<float>(p, luma != nullptr, device, st);
    case FA_F64: return pool_launch<double>(p, luma != nullptr, device, st);
    case FA_U16: return pool_launch<unsigned short>(p, luma != nullptr, device, st);
    default: return FA_E_DTYPE;
  }
}

int box_down_impl(const View& x, int dtype, const double* luma, int f, float* out, int device,
                  cudaStream_t st) {
  if (!x.data || !out) return FA_E_ARG;
  if (f < 2 || f > 64) return FA_E_ARG;
  if (x.n <= 0 || x.c <= 0 || x.h <= 0 || x.w <= 0) return FA_E_SHAPE;
  if (luma && x.c != 3) return FA_E_SHAPE;
  const int pad = f / 2;
  const int hc = x.h + 2 * pad - f + 1, wc = x.w + 2 * pad - f + 1;
  if (hc <= 0 || wc <= 0) return FA_E_SHAPE;
  PoolArgs p{};
  p.x = static_cast<const char*>(x.data);
  p.sn = x.sn; p.sc = x.sc; p.sh = x.sh;
  p.N = x.n; p.C = x.c; p.H = x.h; p.W = x.w;
  p.Cm = luma ? 1 : x.c;
  p.Hp = (hc + f - 1) / f; p.Wp = (wc + f - 1) / f;
  if (luma) {
    p.k0 = (float)luma[0]; p.k1 = (float)luma[1]; p.k2 = (float)luma[2]; p.k3 = (float)luma[3];
  }
  p.out = out;
  const float wgt = (float)(1.0 / ((double)f * f));
  const unsigned g = grid_for((long long)p.N * p.Cm * p.Hp * p.Wp, device);
#define FAB_BOX(T)                                                                    \
  do {                                                                                \
    if (luma) box_down_kernel<T, true><<<g, 256, 0, st>>>(p, f, pad, wgt);            \
    else box_down_kernel<T, false><<<g, 256, 0, st>>>(p, f, pad, wgt);                \
  } while (0)
  switch (dtype) {
    case FA_U8: FAB_BOX(unsigned char); break;
    case FA_F16: FAB_BOX(f16_t); break;
    case FA_BF16: FAB_BOX(bf16_t); break;
    case FA_F32: FAB_BOX(float); break;
    case FA_F64: FAB_BOX(double); break;
    case FA_U16: FAB_BOX(unsigned short); break;
    default: return FA_E_DTYPE;
  }
#undef FAB_BOX
  FAB_LAUNCH_CHECK();
  return FA_OK;
}

int box_down_backward_impl(const float* g, int N, int C, int H, int W, int f, float* dx,
                           int device, cudaStream_t st) {
  if (!g || !dx) return FA_E_ARG;
  if (f < 2 || f > 64) return FA_E_ARG;
  if (N <= 0 || C <= 0 || H <= 0 || W <= 0) return FA_E_SHAPE;
  const int pad = f / 2;
  const int hc = H + 2 * pad - f + 1, wc = W + 2 * pad - f + 1;
  if (hc <= 0 || wc <= 0) return FA_E_SHAPE;
  const int Hp = (hc + f - 1) / f, Wp = (wc + f - 1) / f;
  const long long work = (long long)N * C * H * W;
  box_down_bwd_kernel<<<grid_for(work, device), 256, 0, st>>>(
      g, N * C, H, W, f, pad, Hp, Wp, (float)(1.0 / ((double)f * f)), dx);
  FAB_LAUNCH_CHECK();
  return FA_OK;
}

int pool2_backward_impl(const float* g, int N, int C, int H, int W, float* dx, int device,
                        cudaStream_t st) {
  if (!g || !dx) return FA_E_ARG;
  if (N <= 0 || C <= 0 || H < 2 || W < 2) return FA_E_SHAPE;
  const long long work = (long long)N * C * H * W;
  pool2_bwd_kernel<<<grid_for(work, device), 256, 0, st>>>(g, N * C, H, W, H / 2, W / 2, dx);
  FAB_LAUNCH_CHECK();
  return FA_OK;
}

}  // namespace fab
