// SSIM forward (per-plane SSIM / cs means, map, batch reductions) and the
// fused SSIM backward on sm_100a.
//
// Math (reference: frame_analytics/reference.py:118-160 and the fused kernels
// of fa_cuda.cu:389-784):
//   x' = x - shift, y' = y - shift            (shift = L/2, functional.py:648-650)
//   four Gaussian-blurred planes  E[x'], E[y'], E[x'y'], E[(x'-y')^2]
//   mx = E[x'] + shift, sxy = E[x'y'] - ux*uy,
//   sxx + syy = E[(x'-y')^2] + 2*sxy - (ux - uy)^2
//   S  = (2 mx my + C1)(2 sxy + C2) / ((mx^2 + my^2 + C1)(sxx + syy + C2))
//   cs = (2 sxy + C2) / (sxx + syy + C2)
// Backward (per output position o, upstream g):
//   b = g dS/dsxx, c = g dS/dsxy, t_x = g dS/dmx - 2 b ux - c uy
//   dx(i) = 2 x'(i) (w*b)(i) + y'(i) (w*c)(i) + (w*t_x)(i)    (w* = transposed blur)
//
// Design (B200, FP32-issue bound, no tensor cores):
//   * a block owns a strip of 32*KW columns and streams down a chunk of rows;
//     thread t owns column t;
//   * rows arrive KW at a time; warp k blurs staged row k horizontally, each
//     lane producing KW adjacent columns from 2*KW-1 inputs held in registers
//     (products x'y', (x'-y')^2 formed once per input);
//   * the vertical blur keeps the last KW rows of each column in registers (a
//     ring whose slot index is static because the row loop is unrolled by KW),
//     so each output row costs one shared-memory read per plane instead of KW;
//   * the backward chains moments -> coefficients -> transposed blur -> dx in
//     the same block, so nothing frame-sized is written besides dx / dy;
//   * per-block partials and a last-block finaliser make every forward a single
//     launch with a deterministic reduction order.
#include "common.cuh"

namespace fab {

struct SsimArgs {
  const char* x;
  const char* y;
  long long sn, sc, sh;
  int N, C, H, W;
  int P, Cm;          // planes / channels the metric sees (luma: Cm = 1)
  int Hout, Wout;
  float shift, C1, C2;
  float lk0, lk1, lk2, lk3;
  const float* win;
  int strips, chunks, RH;
  // forward
  float* map_out;
  unsigned int* counter;
  double* part_s;
  double* part_cs;
  double* out_plane_s;
  double* out_plane_cs;
  double* out_per_image;
  double* out_total;
  // backward
  const float* dmap;
  const float* gscalar;
  const float* gs;
  const float* gcs;
  float grad_norm;
  float* dx;
  float* dy;
};

template <int KW>
struct Geo {
  static constexpr int NT = 32 * KW;       // threads; also moment columns per strip
  static constexpr int SW = NT + KW - 1;   // staged input width
  static constexpr int NE = (KW * SW + NT - 1) / NT;  // staged elements per thread
  static constexpr int TD = NT - (KW - 1); // backward: dx columns per strip
};

// Load this thread's share of KW input rows x (SW columns from col0) into
// registers, as shifted floats (luma applied); zero outside the image.
template <typename T, bool LUMA, int KW>
__device__ __forceinline__ void stage_load(const SsimArgs& p, long long base, int row0,
                                           int col0, float (&vx)[Geo<KW>::NE],
                                           float (&vy)[Geo<KW>::NE]) {
  using G = Geo<KW>;
  const T* X = reinterpret_cast<const T*>(p.x);
  const T* Y = reinterpret_cast<const T*>(p.y);
#pragma unroll
  for (int e = 0; e < G::NE; ++e) {
    const int idx = threadIdx.x + e * G::NT;
    const int r = idx / G::SW;
    const int c = idx - r * G::SW;
    const int gr = row0 + r, gc = col0 + c;
    float a = 0.f, b = 0.f;
    if (idx < KW * G::SW && gr >= 0 && gr < p.H && gc >= 0 && gc < p.W) {
      const long long o = base + (long long)gr * p.sh + gc;
      if constexpr (LUMA) {
        a = fmaf(p.lk0, Ld<T>::f(ldro(X + o)),
                 fmaf(p.lk1, Ld<T>::f(ldro(X + o + p.sc)),
                      fmaf(p.lk2, Ld<T>::f(ldro(X + o + 2 * p.sc)), p.lk3)));
        b = fmaf(p.lk0, Ld<T>::f(ldro(Y + o)),
                 fmaf(p.lk1, Ld<T>::f(ldro(Y + o + p.sc)),
                      fmaf(p.lk2, Ld<T>::f(ldro(Y + o + 2 * p.sc)), p.lk3)));
      } else {
        a = Ld<T>::f(ldro(X + o));
        b = Ld<T>::f(ldro(Y + o));
      }
      a -= p.shift;
      b -= p.shift;
    }
    vx[e] = a;
    vy[e] = b;
  }
}

template <int KW>
__device__ __forceinline__ void stage_store(float* sx, float* sy, const float (&vx)[Geo<KW>::NE],
                                            const float (&vy)[Geo<KW>::NE]) {
  using G = Geo<KW>;
#pragma unroll
  for (int e = 0; e < G::NE; ++e) {
    const int idx = threadIdx.x + e * G::NT;
    if (idx < KW * G::SW) {
      sx[idx] = vx[e];
      sy[idx] = vy[e];
    }
  }
}

// Horizontal blur of the four moment planes: KW adjacent outputs from 2KW-1
// staged inputs.  out[o] = sum_j w[j] * plane(q = o + j).
template <int KW>
__device__ __forceinline__ void hblur_moments(const float* __restrict__ sx,
                                              const float* __restrict__ sy,
                                              const float (&w)[KW], float4* __restrict__ out) {
  float4 acc[KW];
#pragma unroll
  for (int o = 0; o < KW; ++o) acc[o] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int q = 0; q < 2 * KW - 1; ++q) {
    const float xv = sx[q], yv = sy[q];
    const float xy = xv * yv;
    const float dv = xv - yv;
    const float dd = dv * dv;
#pragma unroll
    for (int o = 0; o < KW; ++o) {
      const int j = q - o;
      if (j >= 0 && j < KW) {
        acc[o].x = fmaf(w[j], xv, acc[o].x);
        acc[o].y = fmaf(w[j], yv, acc[o].y);
        acc[o].z = fmaf(w[j], xy, acc[o].z);
        acc[o].w = fmaf(w[j], dd, acc[o].w);
      }
    }
  }
#pragma unroll
  for (int o = 0; o < KW; ++o) out[o] = acc[o];
}

// Horizontal blur of NPL coefficient planes (backward scatter).
template <int KW, int NPL>
__device__ __forceinline__ void hblur_coef(const float4* __restrict__ sc,
                                           const float (&w)[KW], float4* __restrict__ out) {
  float4 acc[KW];
#pragma unroll
  for (int o = 0; o < KW; ++o) acc[o] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int q = 0; q < 2 * KW - 1; ++q) {
    const float4 v = sc[q];
#pragma unroll
    for (int o = 0; o < KW; ++o) {
      const int j = q - o;
      if (j >= 0 && j < KW) {
        acc[o].x = fmaf(w[j], v.x, acc[o].x);
        acc[o].y = fmaf(w[j], v.y, acc[o].y);
        acc[o].z = fmaf(w[j], v.z, acc[o].z);
        if (NPL == 4) acc[o].w = fmaf(w[j], v.w, acc[o].w);
      }
    }
  }
#pragma unroll
  for (int o = 0; o < KW; ++o) out[o] = acc[o];
}

// Vertical blur over the register ring: the newest row sits in slot k, the
// output row needs slots k+1 .. k+KW (mod KW), oldest first.
template <int KW, int K, int NPL>
__device__ __forceinline__ float4 vblur(const float4 (&ring)[KW], const float (&w)[KW]) {
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int j = 0; j < KW; ++j) {
    const float4 h = ring[(K + 1 + j) % KW];
    s.x = fmaf(w[j], h.x, s.x);
    s.y = fmaf(w[j], h.y, s.y);
    s.z = fmaf(w[j], h.z, s.z);
    if (NPL == 4) s.w = fmaf(w[j], h.w, s.w);
  }
  return s;
}

template <int KW>
__device__ __forceinline__ void load_taps(const float* win, float (&w)[KW]) {
#pragma unroll
  for (int j = 0; j < KW; ++j) w[j] = __ldg(win + j);
}

// ---------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------
constexpr int FWD_MAP = 1;
constexpr int FWD_CS = 2;

__device__ void ssim_fwd_finalize(const SsimArgs& p, int bpp) {
  __shared__ double s_red[32];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int nw = blockDim.x >> 5;
  const double npix = (double)p.Hout * (double)p.Wout;
  for (int pl = wid; pl < p.P; pl += nw) {
    double s = 0.0, c = 0.0;
    for (int i = lane; i < bpp; i += 32) {
      s += p.part_s[(long long)pl * bpp + i];
      if (p.part_cs) c += p.part_cs[(long long)pl * bpp + i];
    }
    s = warp_sum(s);
    c = warp_sum(c);
    if (lane == 0) {
      p.part_s[(long long)pl * bpp] = s;
      if (p.out_plane_s) p.out_plane_s[pl] = s / npix;
      if (p.out_plane_cs) p.out_plane_cs[pl] = c / npix;
    }
  }
  __syncthreads();
  __threadfence_block();
  double t = 0.0;
  for (int n = threadIdx.x; n < p.N; n += blockDim.x) {
    double s = 0.0;
    for (int c = 0; c < p.Cm; ++c) s += p.part_s[(long long)(n * p.Cm + c) * bpp];
    if (p.out_per_image) p.out_per_image[n] = s / (npix * p.Cm);
    t += s;
  }
  t = block_sum(t, s_red);
  if (threadIdx.x == 0 && p.out_total) *p.out_total = t / (npix * p.Cm * (double)p.N);
}

template <typename T, int KW, int FLAGS, bool LUMA>
__global__ void __launch_bounds__(32 * KW, 1) ssim_fwd_kernel(SsimArgs p) {
  using G = Geo<KW>;
  extern __shared__ float4 smem4[];
  float4* sH = smem4;                                        // [KW][NT]
  float* sX = reinterpret_cast<float*>(smem4 + KW * G::NT);  // [KW][SW]
  float* sY = sX + KW * G::SW;
  __shared__ double s_red[32];
  __shared__ int s_flag;

  const int t = threadIdx.x;
  const int lane = t & 31, warp = t >> 5;
  const int plane = blockIdx.z;
  const int pn = plane / p.Cm, pc = plane - pn * p.Cm;
  const long long base = (long long)pn * p.sn + (long long)pc * p.sc;
  const int c0 = blockIdx.x * G::NT;
  const int r0 = blockIdx.y * p.RH;
  const int rows = min(p.RH, p.Hout - r0);
  const int col = c0 + t;
  const bool col_ok = col < p.Wout;
  const int iters = (rows + KW - 1 + KW - 1) / KW;

  float w[KW];
  load_taps<KW>(p.win, w);

  float vx[G::NE], vy[G::NE];
  stage_load<T, LUMA, KW>(p, base, r0, c0, vx, vy);
  stage_store<KW>(sX, sY, vx, vy);

  float4 ring[KW];
#pragma unroll
  for (int k = 0; k < KW; ++k) ring[k] = make_float4(0.f, 0.f, 0.f, 0.f);
  double acc_s = 0.0, acc_cs = 0.0;
  const long long mbase = (long long)plane * p.Hout * p.Wout;

  for (int m = 0; m < iters; ++m) {
    __syncthreads();
    // horizontal: warp k -> staged row k, lane -> columns [lane*KW, lane*KW+KW)
    hblur_moments<KW>(sX + warp * G::SW + lane * KW, sY + warp * G::SW + lane * KW, w,
                      sH + warp * G::NT + lane * KW);
    __syncthreads();
    const bool more = (m + 1 < iters);
    if (more) stage_load<T, LUMA, KW>(p, base, r0 + (m + 1) * KW, c0, vx, vy);
    // vertical + epilogue
    float fs = 0.f, fcs = 0.f;
#pragma unroll
    for (int k = 0; k < KW; ++k) {
      ring[k] = sH[k * G::NT + t];
      const int o = m * KW + k - (KW - 1);
      if (o >= 0 && o < rows && col_ok) {
        float4 s;
        switch (k) {  // static slot index
#define FAB_VB(KK) case KK: s = vblur<KW, (KK < KW ? KK : 0), 4>(ring, w); break;
          FAB_VB(0) FAB_VB(1) FAB_VB(2) FAB_VB(3) FAB_VB(4) FAB_VB(5)
          FAB_VB(6) FAB_VB(7) FAB_VB(8) FAB_VB(9) FAB_VB(10)
#undef FAB_VB
          default: s = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        const float ux = s.x, uy = s.y;
        const float mx = ux + p.shift, my = uy + p.shift;
        const float sxy = fmaf(-ux, uy, s.z);
        const float du = ux - uy;
        const float sxs = fmaf(-du, du, fmaf(2.f, sxy, s.w));
        const float A1 = fmaf(2.f * mx, my, p.C1);
        const float A2 = fmaf(2.f, sxy, p.C2);
        const float B1 = fmaf(mx, mx, fmaf(my, my, p.C1));
        const float B2 = sxs + p.C2;
        float S;
        if (FLAGS & FWD_CS) {
          const float inv = 1.0f / (B1 * B2);
          S = A1 * A2 * inv;
          fcs += A2 * B1 * inv;
        } else {
          S = (A1 * A2) / (B1 * B2);
        }
        fs += S;
        if (FLAGS & FWD_MAP) p.map_out[mbase + (long long)(r0 + o) * p.Wout + col] = S;
      }
    }
    acc_s += (double)fs;
    acc_cs += (double)fcs;
    if (more) stage_store<KW>(sX, sY, vx, vy);
  }

  // block partials
  const int bpp = p.strips * p.chunks;
  const long long pidx = (long long)plane * bpp + blockIdx.y * p.strips + blockIdx.x;
  acc_s = block_sum(acc_s, s_red);
  if (t == 0) p.part_s[pidx] = acc_s;
  if (FLAGS & FWD_CS) {
    acc_cs = block_sum(acc_cs, s_red);
    if (t == 0) p.part_cs[pidx] = acc_cs;
  }
  if (last_block_arrived(p.counter, gridDim.x * gridDim.y * gridDim.z, &s_flag))
    ssim_fwd_finalize(p, bpp);
}

// ---------------------------------------------------------------------------
// backward
// ---------------------------------------------------------------------------
constexpr int G_MAP = 0;     // dL/dmap per position
constexpr int G_SCALAR = 1;  // dL/d(batch mean), one device scalar
constexpr int G_PLANE = 2;   // dL/d(plane-mean S) and dL/d(plane-mean cs)

template <int KW, bool DX, bool DY, int GMODE>
__global__ void __launch_bounds__(32 * KW, 1) ssim_bwd_kernel(SsimArgs p) {
  using G = Geo<KW>;
  constexpr int NPL = (DX && DY) ? 4 : 3;
  constexpr int SCW = G::NT + KW - 1;  // coefficient row width (zero padded)
  extern __shared__ float4 smem4[];
  float4* sH = smem4;                  // [KW][NT]   moments, then scatter rows
  float4* sC = sH + KW * G::NT;        // [KW][SCW]  coefficients
  float* sX = reinterpret_cast<float*>(sC + KW * SCW);  // [KW][SW]
  float* sY = sX + KW * G::SW;

  const int t = threadIdx.x;
  const int lane = t & 31, warp = t >> 5;
  const int plane = blockIdx.z;
  const long long pbase = (long long)plane * p.H * p.W;
  const int c0 = blockIdx.x * G::TD;      // first dx column of the strip
  const int mc0 = c0 - (KW - 1);          // first moment column
  const int r0 = blockIdx.y * p.RH;       // first dx row of the chunk
  const int rows = min(p.RH, p.H - r0);
  const int i0 = r0 - (KW - 1);           // first input row
  const int iters = (rows + 2 * (KW - 1) + KW - 1) / KW;
  const int q = mc0 + t;                  // this thread's moment column
  const bool q_ok = q >= 0 && q < p.Wout;
  const int dcol = c0 + t;                // this thread's dx column
  const bool d_ok = t < G::TD && dcol < p.W;

  float w[KW];
  load_taps<KW>(p.win, w);

  // zero the coefficient padding columns once
  for (int i = t; i < KW * (SCW - G::NT); i += G::NT) {
    const int r = i / (SCW - G::NT), c = i - r * (SCW - G::NT);
    sC[r * SCW + G::NT + c] = make_float4(0.f, 0.f, 0.f, 0.f);
  }

  float gS = 0.f, gCS = 0.f;
  if (GMODE == G_SCALAR) gS = __ldg(p.gscalar) * p.grad_norm;
  if (GMODE == G_PLANE) {
    gS = __ldg(p.gs + plane) * p.grad_norm;
    gCS = __ldg(p.gcs + plane) * p.grad_norm;
  }

  float vx[G::NE], vy[G::NE];
  stage_load<float, false, KW>(p, pbase, i0, mc0, vx, vy);
  stage_store<KW>(sX, sY, vx, vy);

  float4 ring1[KW], ring2[KW];
#pragma unroll
  for (int k = 0; k < KW; ++k) {
    ring1[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    ring2[k] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  const float* X = reinterpret_cast<const float*>(p.x);
  const float* Y = reinterpret_cast<const float*>(p.y);

  for (int m = 0; m < iters; ++m) {
    __syncthreads();
    hblur_moments<KW>(sX + warp * G::SW + lane * KW, sY + warp * G::SW + lane * KW, w,
                      sH + warp * G::NT + lane * KW);
    __syncthreads();
    const bool more = (m + 1 < iters);
    if (more) stage_load<float, false, KW>(p, pbase, i0 + (m + 1) * KW, mc0, vx, vy);
    // vertical moments -> coefficients
#pragma unroll
    for (int k = 0; k < KW; ++k) {
      ring1[k] = sH[k * G::NT + t];
      const int L = m * KW + k;
      const int o = i0 + L - (KW - 1);  // moment row
      float4 cf = make_float4(0.f, 0.f, 0.f, 0.f);
      if (L >= KW - 1 && o >= 0 && o < p.Hout && q_ok) {
        float4 s;
        switch (k) {
#define FAB_VB(KK) case KK: s = vblur<KW, (KK < KW ? KK : 0), 4>(ring1, w); break;
          FAB_VB(0) FAB_VB(1) FAB_VB(2) FAB_VB(3) FAB_VB(4) FAB_VB(5)
          FAB_VB(6) FAB_VB(7) FAB_VB(8) FAB_VB(9) FAB_VB(10)
#undef FAB_VB
          default: s = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        const float ux = s.x, uy = s.y;
        const float mx = ux + p.shift, my = uy + p.shift;
        const float sxy = fmaf(-ux, uy, s.z);
        const float du = ux - uy;
        const float sxs = fmaf(-du, du, fmaf(2.f, sxy, s.w));
        const float A1 = fmaf(2.f * mx, my, p.C1);
        const float A2 = fmaf(2.f, sxy, p.C2);
        const float B1 = fmaf(mx, mx, fmaf(my, my, p.C1));
        const float B2 = sxs + p.C2;
        const float iB1 = 1.0f / B1;
        const float iB2 = 1.0f / B2;
        const float S = A1 * A2 * iB1 * iB2;
        const float kk = 2.f * A2 * iB1 * iB2;
        float g = gS, bb, cc;
        if (GMODE == G_MAP) g = __ldg(p.dmap + (long long)plane * p.Hout * p.Wout + (long long)o * p.Wout + q);
        if (GMODE == G_PLANE) {
          const float CS = A2 * iB2;
          bb = -(g * S + gCS * CS) * iB2;
          cc = 2.f * (g * A1 * iB1 + gCS) * iB2;
        } else {
          bb = -g * S * iB2;
          cc = 2.f * g * A1 * iB1 * iB2;
        }
        const float tx = g * kk * (my - mx * A1 * iB1) - 2.f * bb * ux - cc * uy;
        const float ty = g * kk * (mx - my * A1 * iB1) - 2.f * bb * uy - cc * ux;
        cf.x = bb;
        cf.y = cc;
        if (DX && DY) { cf.z = tx; cf.w = ty; }
        else cf.z = DX ? tx : ty;
      }
      sC[k * SCW + t] = cf;
    }
    __syncthreads();
    // horizontal scatter of the coefficient rows
    hblur_coef<KW, NPL>(sC + warp * SCW + lane * KW, w, sH + warp * G::NT + lane * KW);
    __syncthreads();
    // vertical scatter -> dx, dy
#pragma unroll
    for (int k = 0; k < KW; ++k) {
      ring2[k] = sH[k * G::NT + t];
      const int L = m * KW + k;
      const int r = i0 + L - (KW - 1);  // dx row
      if (L >= 2 * (KW - 1) && r < r0 + rows && d_ok) {
        float4 s;
        switch (k) {
#define FAB_VB(KK) case KK: s = vblur<KW, (KK < KW ? KK : 0), NPL>(ring2, w); break;
          FAB_VB(0) FAB_VB(1) FAB_VB(2) FAB_VB(3) FAB_VB(4) FAB_VB(5)
          FAB_VB(6) FAB_VB(7) FAB_VB(8) FAB_VB(9) FAB_VB(10)
#undef FAB_VB
          default: s = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        const long long off = pbase + (long long)r * p.W + dcol;
        const float xs = __ldg(X + off) - p.shift;
        const float ys = __ldg(Y + off) - p.shift;
        if (DX) p.dx[off] = fmaf(2.f * xs, s.x, fmaf(ys, s.y, s.z));
        if (DY) p.dy[off] = fmaf(2.f * ys, s.x, fmaf(xs, s.y, (DX && DY) ? s.w : s.z));
      }
    }
    if (more) stage_store<KW>(sX, sY, vx, vy);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

template <int KW>
static constexpr size_t fwd_smem() {
  return sizeof(float4) * KW * Geo<KW>::NT + sizeof(float) * 2 * KW * Geo<KW>::SW;
}
template <int KW>
static constexpr size_t bwd_smem() {
  return sizeof(float4) * KW * Geo<KW>::NT + sizeof(float4) * KW * (Geo<KW>::NT + KW - 1) +
         sizeof(float) * 2 * KW * Geo<KW>::SW;
}

// cudaFuncSetAttribute once per (kernel, device): `done` must belong to one
// kernel, so each launch_* instantiation passes its own flag array.
template <typename K>
static cudaError_t ensure_smem(K* kern, size_t bytes, int device, bool (&done)[64]) {
  if (device >= 0 && device < 64 && done[device]) return cudaSuccess;
  const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)bytes);
  if (e == cudaSuccess && device >= 0 && device < 64) done[device] = true;
  return e;
}

struct SsimPlan {
  int strips, chunks, RH;
};

static SsimPlan plan_rows(int rows_total, int strips, int planes, int device) {
  const int sms = sm_count(device);
  long long want = (4LL * sms + (long long)strips * planes - 1) / ((long long)strips * planes);
  if (want < 1) want = 1;
  if (want > rows_total) want = rows_total;
  SsimPlan pl;
  pl.strips = strips;
  pl.RH = (int)((rows_total + want - 1) / want);
  pl.chunks = (rows_total + pl.RH - 1) / pl.RH;
  return pl;
}

static SsimPlan fwd_plan(int Hout, int Wout, int K, int planes, int device) {
  const int nt = 32 * K;
  return plan_rows(Hout, (Wout + nt - 1) / nt, planes, device);
}

size_t ssim_ws_bytes(int planes, int Hout, int Wout, int K, int device) {
  const SsimPlan pl = fwd_plan(Hout, Wout, K, planes, device);
  return FAB_COUNTER_BYTES + 2 * sizeof(double) * (size_t)planes * pl.strips * pl.chunks;
}

template <typename T, int KW, int FLAGS, bool LUMA>
static int launch_fwd(SsimArgs& p, int device, cudaStream_t st) {
  auto kern = ssim_fwd_kernel<T, KW, FLAGS, LUMA>;
  const size_t sm = fwd_smem<KW>();
  static bool done[64] = {false};
  FAB_TRY(ensure_smem(kern, sm, device, done));
  dim3 grid(p.strips, p.chunks, p.P);
  kern<<<grid, 32 * KW, sm, st>>>(p);
  FAB_LAUNCH_CHECK();
  return FA_OK;
}

template <typename T, int FLAGS, bool LUMA>
static int fwd_k(SsimArgs& p, int K, int device, cudaStream_t st) {
  switch (K) {
    case 11: return launch_fwd<T, 11, FLAGS, LUMA>(p, device, st);
    case 9: return launch_fwd<T, 9, FLAGS, LUMA>(p, device, st);
    case 7: return launch_fwd<T, 7, FLAGS, LUMA>(p, device, st);
    case 5: return launch_fwd<T, 5, FLAGS, LUMA>(p, device, st);
    case 3: return launch_fwd<T, 3, FLAGS, LUMA>(p, device, st);
    default: return FA_E_WINDOW;
  }
}

template <typename T, bool LUMA>
static int fwd_flags(SsimArgs& p, int K, int device, cudaStream_t st) {
  const int flags = (p.map_out ? FWD_MAP : 0) | ((p.out_plane_cs) ? FWD_CS : 0);
  switch (flags) {
    case 0: return fwd_k<T, 0, LUMA>(p, K, device, st);
    case FWD_MAP: return fwd_k<T, FWD_MAP, LUMA>(p, K, device, st);
    case FWD_CS: return fwd_k<T, FWD_CS, LUMA>(p, K, device, st);
    default: return fwd_k<T, FWD_MAP | FWD_CS, LUMA>(p, K, device, st);
  }
}

template <typename T>
static int fwd_luma(SsimArgs& p, bool luma, int K, int device, cudaStream_t st) {
  return luma ? fwd_flags<T, true>(p, K, device, st) : fwd_flags<T, false>(p, K, device, st);
}

int ssim_fwd_impl(const View& x, const View& y, int dtype, const double* luma,
                  const float* win, int K, double shift, double C1, double C2,
                  float* map_out, void* ws, size_t ws_bytes, double* out_plane_s,
                  double* out_plane_cs, double* out_per_image, double* out_total,
                  int device, cudaStream_t st) {
  if (!x.data || !y.data || !win || !ws) return FA_E_ARG;
  if (x.n <= 0 || x.c <= 0 || x.h <= 0 || x.w <= 0) return FA_E_SHAPE;
  if (x.n != y.n || x.c != y.c || x.h != y.h || x.w != y.w) return FA_E_SHAPE;
  if (x.sn != y.sn || x.sc != y.sc || x.sh != y.sh) return FA_E_SHAPE;
  if (K < 3 || K > FA_MAX_WIN || (K & 1) == 0) return FA_E_WINDOW;
  if (luma && x.c != 3) return FA_E_SHAPE;
  const int Hout = x.h - K + 1, Wout = x.w - K + 1;
  if (Hout <= 0 || Wout <= 0) return FA_E_SHAPE;
  SsimArgs p{};
  p.x = static_cast<const char*>(x.data);
  p.y = static_cast<const char*>(y.data);
  p.sn = x.sn; p.sc = x.sc; p.sh = x.sh;
  p.N = x.n; p.C = x.c; p.H = x.h; p.W = x.w;
  p.Cm = luma ? 1 : x.c;
  p.P = p.N * p.Cm;
  if (p.P > 65535) return FA_E_SHAPE;
  p.Hout = Hout; p.Wout = Wout;
  p.shift = (float)shift; p.C1 = (float)C1; p.C2 = (float)C2;
  if (luma) {
    p.lk0 = (float)luma[0]; p.lk1 = (float)luma[1]; p.lk2 = (float)luma[2]; p.lk3 = (float)luma[3];
  }
  p.win = win;
  const SsimPlan pl = fwd_plan(Hout, Wout, K, p.P, device);
  p.strips = pl.strips; p.chunks = pl.chunks; p.RH = pl.RH;
  const size_t nb = (size_t)p.P * pl.strips * pl.chunks;
  if (ws_bytes < FAB_COUNTER_BYTES + 2 * sizeof(double) * nb) return FA_E_ARG;
  p.counter = static_cast<unsigned int*>(ws);
  p.part_s = reinterpret_cast<double*>(static_cast<char*>(ws) + FAB_COUNTER_BYTES);
  p.part_cs = p.part_s + nb;
  p.map_out = map_out;
  p.out_plane_s = out_plane_s; p.out_plane_cs = out_plane_cs;
  p.out_per_image = out_per_image; p.out_total = out_total;
  if (!out_plane_cs) p.part_cs = nullptr;
  switch (dtype) {
    case FA_U8: return fwd_luma<unsigned char>(p, luma != nullptr, K, device, st);
    case FA_F16: return fwd_luma<f16_t>(p, luma != nullptr, K, device, st);
    case FA_BF16: return fwd_luma<bf16_t>(p, luma != nullptr, K, device, st);
    case FA_F32: return fwd_luma<float>(p, luma != nullptr, K, device, st);
    case FA_F64: return fwd_luma<double>(p, luma != nullptr, K, device, st);
    default: return FA_E_DTYPE;
  }
}

template <int KW, bool DX, bool DY, int GMODE>
static int launch_bwd(SsimArgs& p, int device, cudaStream_t st) {
  auto kern = ssim_bwd_kernel<KW, DX, DY, GMODE>;
  const size_t sm = bwd_smem<KW>();
  static bool done[64] = {false};
  FAB_TRY(ensure_smem(kern, sm, device, done));
  dim3 grid(p.strips, p.chunks, p.P);
  kern<<<grid, 32 * KW, sm, st>>>(p);
  FAB_LAUNCH_CHECK();
  return FA_OK;
}

template <bool DX, bool DY, int GMODE>
static int bwd_k(SsimArgs& p, int K, int device, cudaStream_t st) {
  switch (K) {
    case 11: return launch_bwd<11, DX, DY, GMODE>(p, device, st);
    case 9: return launch_bwd<9, DX, DY, GMODE>(p, device, st);
    case 7: return launch_bwd<7, DX, DY, GMODE>(p, device, st);
    case 5: return launch_bwd<5, DX, DY, GMODE>(p, device, st);
    case 3: return launch_bwd<3, DX, DY, GMODE>(p, device, st);
    default: return FA_E_WINDOW;
  }
}

template <int GMODE>
static int bwd_g(SsimArgs& p, int K, int device, cudaStream_t st) {
  if (p.dx && p.dy) return bwd_k<true, true, GMODE>(p, K, device, st);
  if (p.dx) return bwd_k<true, false, GMODE>(p, K, device, st);
  return bwd_k<false, true, GMODE>(p, K, device, st);
}

int ssim_bwd_impl(const float* x, const float* y, int N, int C, int H, int W,
                  const float* win, int K, double shift, double C1, double C2,
                  const float* dmap, const float* gscalar, const float* gs,
                  const float* gcs, float* dx, float* dy, int device, cudaStream_t st) {
  if (!x || !y || !win) return FA_E_ARG;
  if (!dx && !dy) return FA_E_ARG;
  const int forms = (dmap ? 1 : 0) + (gscalar ? 1 : 0) + ((gs || gcs) ? 1 : 0);
  if (forms != 1) return FA_E_ARG;
  if ((gs != nullptr) != (gcs != nullptr)) return FA_E_ARG;
  if (N <= 0 || C <= 0 || H <= 0 || W <= 0) return FA_E_SHAPE;
  if (K < 3 || K > FA_MAX_WIN || (K & 1) == 0) return FA_E_WINDOW;
  const int Hout = H - K + 1, Wout = W - K + 1;
  if (Hout <= 0 || Wout <= 0) return FA_E_SHAPE;
  SsimArgs p{};
  p.x = reinterpret_cast<const char*>(x);
  p.y = reinterpret_cast<const char*>(y);
  p.N = N; p.C = C; p.H = H; p.W = W;
  p.Cm = C; p.P = N * C;
  if (p.P > 65535) return FA_E_SHAPE;
  p.sn = (long long)C * H * W; p.sc = (long long)H * W; p.sh = W;
  p.Hout = Hout; p.Wout = Wout;
  p.shift = (float)shift; p.C1 = (float)C1; p.C2 = (float)C2;
  p.win = win;
  p.dmap = dmap; p.gscalar = gscalar; p.gs = gs; p.gcs = gcs;
  p.dx = dx; p.dy = dy;
  const double npix = (double)Hout * Wout;
  p.grad_norm = gscalar ? (float)(1.0 / (npix * p.P)) : (gs ? (float)(1.0 / npix) : 1.0f);
  const int td = 32 * K - (K - 1);
  const SsimPlan pl = plan_rows(H, (W + td - 1) / td, p.P, device);
  p.strips = pl.strips; p.chunks = pl.chunks; p.RH = pl.RH;
  if (dmap) return bwd_g<G_MAP>(p, K, device, st);
  if (gscalar) return bwd_g<G_SCALAR>(p, K, device, st);
  return bwd_g<G_PLANE>(p, K, device, st);
}

}  // namespace fab
