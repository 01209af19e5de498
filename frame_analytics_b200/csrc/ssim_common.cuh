// Shared pieces of the SSIM forward and backward kernels (sm_100a).
//
// Math (reference: frame_analytics/reference.py:118-160 and the fused kernels
// of fa_cuda.cu:389-784):
//   x' = x - shift, y' = y - shift            (shift = L/2, functional.py:648-650)
//   four Gaussian-blurred planes  E[x'], E[y'], E[x'y'], E[(x'-y')^2]
//   mx = E[x'] + shift, sxy = E[x'y'] - ux*uy,
//   sxx + syy = E[(x'-y')^2] + 2*sxy - (ux - uy)^2
//   S  = (2 mx my + C1)(2 sxy + C2) / ((mx^2 + my^2 + C1)(sxx + syy + C2))
//   cs = (2 sxy + C2) / (sxx + syy + C2)
//
// Layout (B200; the path is FP32-issue bound, so the design minimises
// instructions per pixel and keeps every warp issuing):
//   * a block owns a strip of 32*KW columns and streams down a chunk of rows;
//     thread t owns column t of the vertical pass;
//   * rows arrive KW at a time, copied global->shared with cp.async (no
//     registers, no stall) and converted in place to shifted floats;
//   * warp k blurs staged row k horizontally, each lane producing KW adjacent
//     columns from 2*KW-1 staged inputs held in registers; the (x', y') planes
//     and the product planes (x'y', (x'-y')^2) are two passes, which halves the
//     live accumulators;
//   * the vertical blur keeps the last KW rows of its column in registers (a
//     ring whose slot index is static because the row loop is unrolled by KW),
//     so an output row costs one 16-byte shared load instead of KW;
//   * the Gaussian taps travel in the kernel parameters, so every FMA reads
//     its tap from the constant bank instead of a register.
#pragma once

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
  float w[12];        // Gaussian taps
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
  static constexpr int NT = 32 * KW;                   // threads = moment columns per strip
  static constexpr int SW = NT + KW - 1;               // staged input width
  static constexpr int NE = (KW * SW + NT - 1) / NT;   // staged elements per thread
  static constexpr int TD = NT - (KW - 1);             // backward: dx columns per strip
};

// Staging modes: cp.async of raw elements (aligned views, no luma), register
// loads of any strided view, and register loads with the luma projection.
constexpr int STAGE_ASYNC = 0;
constexpr int STAGE_GENERIC = 1;
constexpr int STAGE_LUMA = 2;

// raw-staging geometry for cp.async: 4-byte chunks (8 for float64)
template <typename T, int KW>
struct Raw {
  static constexpr int CB = sizeof(T) == 8 ? 8 : 4;     // bytes per copy
  static constexpr int EPC = CB / (int)sizeof(T);        // elements per copy
  static constexpr int RC = (Geo<KW>::SW + EPC - 1) / EPC;  // copies per row
  static constexpr int RPE = RC * EPC;                   // raw row pitch, elements
  static constexpr bool kInPlace = std::is_same<T, float>::value;
  static constexpr size_t kBytes = kInPlace ? 0 : sizeof(T) * 2 * KW * RPE;
};

// ---------------------------------------------------------------------------
// cp.async
// ---------------------------------------------------------------------------
template <int CB>
__device__ __forceinline__ void cp_async(void* smem, const void* gmem, int src_bytes) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  if constexpr (CB == 8) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;\n" ::"r"(s), "l"(gmem),
                 "r"(src_bytes));
  } else {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(s), "l"(gmem),
                 "r"(src_bytes));
  }
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// Issue the copies of KW rows (SW columns from col0) of one plane.  Rows and
// columns outside the image are zero-filled (their values feed only outputs
// that are never used).
template <typename T, int KW>
__device__ __forceinline__ void stage_async(const SsimArgs& p, long long base, int row0,
                                            int col0, T* rawx, T* rawy) {
  using R = Raw<T, KW>;
  const T* X = reinterpret_cast<const T*>(p.x) + base;
  const T* Y = reinterpret_cast<const T*>(p.y) + base;
  for (int i = threadIdx.x; i < KW * R::RC; i += Geo<KW>::NT) {
    const int r = i / R::RC;
    const int ch = i - r * R::RC;
    const int gr = row0 + r, gc = col0 + ch * R::EPC;
    int nb = 0;
    long long off = 0;
    if (gr >= 0 && gr < p.H && gc >= 0 && gc < p.W) {
      nb = min(R::CB, (p.W - gc) * (int)sizeof(T));
      off = (long long)gr * p.sh + gc;
    }
    cp_async<R::CB>(rawx + r * R::RPE + ch * R::EPC, X + off, nb);
    cp_async<R::CB>(rawy + r * R::RPE + ch * R::EPC, Y + off, nb);
  }
  cp_async_commit();
}

// After the copies landed: this thread's own chunks -> shifted floats.
template <typename T, int KW>
__device__ __forceinline__ void stage_convert(const SsimArgs& p, const T* rawx, const T* rawy,
                                              float* sx, float* sy) {
  using R = Raw<T, KW>;
  using G = Geo<KW>;
  for (int i = threadIdx.x; i < KW * R::RC; i += G::NT) {
    const int r = i / R::RC;
    const int ch = i - r * R::RC;
#pragma unroll
    for (int e = 0; e < R::EPC; ++e) {
      const int c = ch * R::EPC + e;
      if (c < G::SW) {
        sx[r * G::SW + c] = Ld<T>::f(rawx[r * R::RPE + c]) - p.shift;
        sy[r * G::SW + c] = Ld<T>::f(rawy[r * R::RPE + c]) - p.shift;
      }
    }
  }
}

// Register staging (strided or luma views): load converted values ...
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

// ... and store them once the buffer is free.
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

// ---------------------------------------------------------------------------
// blurs
// ---------------------------------------------------------------------------

// Horizontal blur of the (x', y') planes: KW adjacent outputs from 2KW-1
// staged inputs; out[o].xy = sum_j w[j] * plane(o + j).
template <int KW>
__device__ __forceinline__ void hblur_xy(const SsimArgs& p, const float* __restrict__ sx,
                                         const float* __restrict__ sy, float4* __restrict__ out) {
  float2 acc[KW];
#pragma unroll
  for (int o = 0; o < KW; ++o) acc[o] = make_float2(0.f, 0.f);
#pragma unroll
  for (int q = 0; q < 2 * KW - 1; ++q) {
    const float xv = sx[q], yv = sy[q];
#pragma unroll
    for (int o = 0; o < KW; ++o) {
      const int j = q - o;
      if (j >= 0 && j < KW) {
        acc[o].x = fmaf(p.w[j], xv, acc[o].x);
        acc[o].y = fmaf(p.w[j], yv, acc[o].y);
      }
    }
  }
#pragma unroll
  for (int o = 0; o < KW; ++o) reinterpret_cast<float2*>(out + o)[0] = acc[o];
}

// Horizontal blur of the product planes (x'y', (x'-y')^2) -> out[o].zw.
template <int KW>
__device__ __forceinline__ void hblur_prod(const SsimArgs& p, const float* __restrict__ sx,
                                           const float* __restrict__ sy,
                                           float4* __restrict__ out) {
  float2 acc[KW];
#pragma unroll
  for (int o = 0; o < KW; ++o) acc[o] = make_float2(0.f, 0.f);
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
        acc[o].x = fmaf(p.w[j], xy, acc[o].x);
        acc[o].y = fmaf(p.w[j], dd, acc[o].y);
      }
    }
  }
#pragma unroll
  for (int o = 0; o < KW; ++o) reinterpret_cast<float2*>(out + o)[1] = acc[o];
}

// Horizontal blur of two float components of float4 rows (backward scatter).
// HALF selects .xy (0) or .zw (1); NC = 1 blurs only the first of the pair.
template <int KW, int HALF, int NC>
__device__ __forceinline__ void hblur_pair(const SsimArgs& p, const float4* __restrict__ sc,
                                           float4* __restrict__ out) {
  float2 acc[KW];
#pragma unroll
  for (int o = 0; o < KW; ++o) acc[o] = make_float2(0.f, 0.f);
#pragma unroll
  for (int q = 0; q < 2 * KW - 1; ++q) {
    const float2 v = reinterpret_cast<const float2*>(sc + q)[HALF];
#pragma unroll
    for (int o = 0; o < KW; ++o) {
      const int j = q - o;
      if (j >= 0 && j < KW) {
        acc[o].x = fmaf(p.w[j], v.x, acc[o].x);
        if (NC == 2) acc[o].y = fmaf(p.w[j], v.y, acc[o].y);
      }
    }
  }
#pragma unroll
  for (int o = 0; o < KW; ++o) reinterpret_cast<float2*>(out + o)[HALF] = acc[o];
}

// Vertical blur over the register ring: the newest row sits in slot K, the
// output row needs slots K+1 .. K+KW (mod KW), oldest first.
template <int KW, int K, int NPL>
__device__ __forceinline__ float4 vblur(const SsimArgs& p, const float4 (&ring)[KW]) {
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int j = 0; j < KW; ++j) {
    const float4 h = ring[(K + 1 + j) % KW];
    s.x = fmaf(p.w[j], h.x, s.x);
    s.y = fmaf(p.w[j], h.y, s.y);
    s.z = fmaf(p.w[j], h.z, s.z);
    if (NPL == 4) s.w = fmaf(p.w[j], h.w, s.w);
  }
  return s;
}

// Static-slot dispatch of vblur for a loop index k that the unroller resolves.
template <int KW, int NPL>
__device__ __forceinline__ float4 vblur_at(const SsimArgs& p, const float4 (&ring)[KW], int k) {
  switch (k) {
#define FAB_VB(KK) \
  case KK: return vblur<KW, (KK < KW ? KK : 0), NPL>(p, ring);
    FAB_VB(0) FAB_VB(1) FAB_VB(2) FAB_VB(3) FAB_VB(4) FAB_VB(5)
    FAB_VB(6) FAB_VB(7) FAB_VB(8) FAB_VB(9) FAB_VB(10)
#undef FAB_VB
    default: return make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

// Local statistics from the four blurred planes.
struct Moments {
  float ux, uy, mx, my, A1, A2, B1, B2;
};

__device__ __forceinline__ Moments moments(const SsimArgs& p, const float4& s) {
  Moments m;
  m.ux = s.x;
  m.uy = s.y;
  m.mx = s.x + p.shift;
  m.my = s.y + p.shift;
  const float sxy = fmaf(-s.x, s.y, s.z);
  const float du = s.x - s.y;
  const float sxs = fmaf(-du, du, fmaf(2.f, sxy, s.w));
  m.A1 = fmaf(2.f * m.mx, m.my, p.C1);
  m.A2 = fmaf(2.f, sxy, p.C2);
  m.B1 = fmaf(m.mx, m.mx, fmaf(m.my, m.my, p.C1));
  m.B2 = sxs + p.C2;
  return m;
}

// cudaFuncSetAttribute once per (kernel, device); each launch instantiation
// owns its `done` flags.
template <typename K>
static cudaError_t ensure_smem(K* kern, size_t bytes, int device, bool (&done)[64]) {
  if (device >= 0 && device < 64 && done[device]) return cudaSuccess;
  const cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e == cudaSuccess && device >= 0 && device < 64) done[device] = true;
  return e;
}

struct SsimPlan {
  int strips, chunks, RH;
};

// Split rows so that the grid holds about `waves` x SMs x blocks-per-SM blocks.
static inline SsimPlan plan_rows(int rows_total, int strips, int planes, int device,
                                 int blocks_per_sm, int waves) {
  const int sms = sm_count(device);
  const long long target = (long long)waves * sms * blocks_per_sm;
  const long long per = (long long)strips * planes;
  long long want = (target + per - 1) / per;
  if (want < 1) want = 1;
  if (want > rows_total) want = rows_total;
  SsimPlan pl;
  pl.strips = strips;
  pl.RH = (int)((rows_total + want - 1) / want);
  pl.chunks = (rows_total + pl.RH - 1) / pl.RH;
  return pl;
}

}  // namespace fab
