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

#include <cuda.h>

#include "common.cuh"

namespace fab {

struct SsimArgs {
  CUtensorMap tmx, tmy;  // TMA row maps of x and y (STAGE_TMA)
  int sofs;              // staged-row offset of the strip's first column
  int tma_d;             // leading elements the aligned map base adds
  const char* x;
  const char* y;
  long long sn, sc, sh;
  int N, C, H, W;
  int P, Cm;          // planes / channels the metric sees (luma: Cm = 1)
  int Hout, Wout;
  float shift, C1, C2;
  float lk0, lk1, lk2, lk3;
  float w[12];        // Gaussian taps
  float2 w2[12];      // the same taps as {w, w} pairs for packed f32x2 FMAs
  int strips, chunks, RH;
  int sym;            // the taps are symmetric: w[j] == w[K-1-j]
  // forward
  float* map_out;
  unsigned int* counter;
  double* part_s;
  double* part_cs;
  double* out_plane_s;
  double* out_plane_cs;
  double* out_per_image;
  double* out_total;
  // fused squared-difference sums (SSIM with MSE / PSNR from the same read)
  void* part_sq;                       // [P][bpp] uint64 (uint8 input) or double
  double psnr_bias;
  double* out_mse_per_image;
  double* out_mse_total;
  double* out_psnr_per_image;
  double* out_psnr_total;
  unsigned long long* out_ssd_per_image;  // uint8 input: exact sums
  // backward
  const float* dmap;
  const float* gscalar;
  const float* gs;
  const float* gcs;
  float grad_norm;
  unsigned int* err;  // host-mapped error word of the bounded waits
  const float* wdev;  // device taps (reference-compatible calls), else null
  // fused GMSD (2x2 pool, Prewitt, pooled over the image's planes)
  float gT, geps;     // threshold and epsilon in the metric's units
  int gHo, gWo;       // GMS map size, (H/2 - 2) x (W/2 - 2)
  double* part_g;     // [P][bpp] (sum d, sum d^2), d = q - 1
  double* out_gms_per_image;
  double* out_gmsd_per_image;
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

// Staging modes: TMA row copies of raw elements (16-byte-compatible views, no
// luma), register loads of any strided view, and register loads with the
// luma projection.
constexpr int STAGE_TMA = 0;
constexpr int STAGE_GENERIC = 1;
constexpr int STAGE_LUMA = 2;

// TMA staging geometry.  Each staged row is two boxes of BW elements landing
// back to back, so a row is contiguous in shared memory.  The first column is
// rounded down to a 16-byte boundary (the TMA x coordinate must be), which
// leaves up to 16/sizeof(T)-1 leading elements: RP = 2*BW covers them.  BW is
// a multiple of 128 bytes so every row half starts 128-byte aligned.
template <typename T, int KW>
struct Raw {
  static constexpr int E = (int)sizeof(T);
  static constexpr int XA = 16 / E;                               // x alignment, elements
  static constexpr int Q = 128 / E;                               // BW granule, elements
  static constexpr int BW = ((Geo<KW>::SW + XA - 1 + 1) / 2 + Q - 1) / Q * Q;
  static constexpr int RP = 2 * BW;                               // raw row pitch, elements
  static constexpr bool kInPlace = std::is_same<T, float>::value;
  // converted-row pitch: float32 converts in place; other types pack tighter
  static constexpr int FP = kInPlace ? RP : (Geo<KW>::SW + XA - 1 + 3) / 4 * 4;
  static constexpr size_t kFloatBytes = (sizeof(float) * 2 * KW * FP + 127) / 128 * 128;  // x, y
  static constexpr size_t kRawBytes = kInPlace ? 0 : (size_t)E * 2 * KW * RP;
  static constexpr unsigned kTxBytes = (unsigned)E * 2u * KW * RP;    // per iteration
  static_assert(BW <= 256, "TMA box too wide");
};

// ---------------------------------------------------------------------------
// TMA + mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ unsigned smem_u32(const void* p) {
  return static_cast<unsigned>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(unsigned long long* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(unsigned long long* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try(unsigned a, unsigned parity) {
  unsigned done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(a), "r"(parity)
      : "memory");
  return done != 0;
}
__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Slow path of a bounded wait: polls until the phase completes, `limit_ns`
// of wall time passes, or another wait has already failed (the error word is
// set).  On giving up it records FA_E_TIMEOUT in the error word, which the
// next call of any entry point turns into its return status, and returns so
// that the kernel finishes instead of hanging; its outputs are then garbage
// and reported as such.  `err` is a host-mapped word (it may be null: the
// wait then only gives up).
static __device__ __noinline__ void mbar_wait_slow(unsigned a, unsigned parity, unsigned* err,
                                            unsigned long long limit_ns) {
  const unsigned long long t0 = globaltimer_ns();
  for (unsigned i = 1;; ++i) {
    if (mbar_try(a, parity)) return;
    if ((i & 255u) == 0u) {
      const bool failed = err && *reinterpret_cast<volatile unsigned*>(err) != 0u;
      if (failed || globaltimer_ns() - t0 > limit_ns) {
        if (err) {
          *reinterpret_cast<volatile unsigned*>(err) = (unsigned)FA_E_TIMEOUT;
          __threadfence_system();
        }
        return;
      }
    }
  }
}
// Bounded wait on a phase: a few fast polls, then the timed slow path (two
// seconds: a row copy takes microseconds).
constexpr unsigned long long kWaitLimitNs = 2000000000ull;
__device__ __forceinline__ void mbar_wait(unsigned long long* bar, unsigned parity,
                                          unsigned* err) {
  const unsigned a = smem_u32(bar);
#pragma unroll 1
  for (int i = 0; i < 32; ++i)
    if (mbar_try(a, parity)) return;
  mbar_wait_slow(a, parity, err, kWaitLimitNs);
}
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}
// One box {BW, 1, 1, 1} of a 4-D map (x, row, channel, image) into smem.
__device__ __forceinline__ void tma_row(void* dst, const CUtensorMap* map, int x, int y, int c,
                                        int n, unsigned long long* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];\n" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<unsigned long long>(map)), "r"(x), "r"(y), "r"(c), "r"(n),
      "r"(smem_u32(bar))
      : "memory");
}

// Warp 0 issues the copies of KW rows of x and y starting at row0: lane r
// copies row r of x, lane 16 + r row r of y (two boxes each), after lane 0 has
// armed the barrier with the byte count.  Rows and columns outside the image
// arrive as zeros.  x0 is the 16-byte-aligned map x coordinate of the strip.
template <typename T, int KW>
__device__ __forceinline__ void stage_tma(const SsimArgs& p, int pn, int pc, int row0, int x0,
                                          T* rawx, T* rawy, unsigned long long* bar) {
  using R = Raw<T, KW>;
  static_assert(KW <= 16, "one lane per row");
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    const int r = lane & 15;
    if (lane == 0) {
      fence_async_smem();  // earlier generic accesses of the buffers come first
      mbar_expect_tx(bar, R::kTxBytes);
    }
    __syncwarp();
    if (r < KW) {
      if (lane != 0) fence_async_smem();
      const CUtensorMap* map = lane < 16 ? &p.tmx : &p.tmy;
      T* dst = (lane < 16 ? rawx : rawy) + r * R::RP;
      tma_row(dst, map, x0, row0 + r, pc, pn, bar);
      tma_row(dst + R::BW, map, x0 + R::BW, row0 + r, pc, pn, bar);
    }
  }
}

// After the copies landed: raw (pitch RP) -> shifted floats (pitch FP), 4
// elements per step.
template <typename T, int KW, bool UV = false>
__device__ __forceinline__ void stage_convert(const SsimArgs& p, const T* rawx, const T* rawy,
                                              float* sx, float* sy) {
  using R = Raw<T, KW>;
  constexpr int N4 = KW * R::RP / 4;
  constexpr int R4 = R::RP / 4;
  for (int i = threadIdx.x; i < N4; i += Geo<KW>::NT) {
    const int r = i / R4, c4 = i - r * R4;
    if (4 * c4 >= R::FP) continue;
    const int o4 = (r * R::FP) / 4 + c4;
    float4 a, b;
    if constexpr (std::is_same<T, float>::value) {
      a = reinterpret_cast<const float4*>(rawx)[i];
      b = reinterpret_cast<const float4*>(rawy)[i];
    } else if constexpr (std::is_same<T, unsigned char>::value) {
      // each byte under 2^23's exponent bits is 2^23 + byte exactly: one
      // byte permute per value and two packed subtracts per pair, no I2F
      const unsigned u = reinterpret_cast<const unsigned*>(rawx)[i];
      const unsigned v = reinterpret_cast<const unsigned*>(rawy)[i];
      constexpr unsigned M = 0x4B000000u;
      const float2 off = make_float2(-8388608.f, -8388608.f), sh = make_float2(-p.shift, -p.shift);
      float2 q[4];
      q[0] = make_float2(__uint_as_float(__byte_perm(u, M, 0x7440)),
                         __uint_as_float(__byte_perm(u, M, 0x7441)));
      q[1] = make_float2(__uint_as_float(__byte_perm(u, M, 0x7442)),
                         __uint_as_float(__byte_perm(u, M, 0x7443)));
      q[2] = make_float2(__uint_as_float(__byte_perm(v, M, 0x7440)),
                         __uint_as_float(__byte_perm(v, M, 0x7441)));
      q[3] = make_float2(__uint_as_float(__byte_perm(v, M, 0x7442)),
                         __uint_as_float(__byte_perm(v, M, 0x7443)));
#pragma unroll
      for (int k = 0; k < 4; ++k) q[k] = __fadd2_rn(__fadd2_rn(q[k], off), sh);
      if constexpr (UV) {
        const float2 m1 = make_float2(-1.f, -1.f);
        const float2 u0 = __fadd2_rn(q[0], q[2]), u1 = __fadd2_rn(q[1], q[3]);
        q[2] = __ffma2_rn(q[2], m1, q[0]);
        q[3] = __ffma2_rn(q[3], m1, q[1]);
        q[0] = u0;
        q[1] = u1;
      }
      reinterpret_cast<float4*>(sx)[o4] = make_float4(q[0].x, q[0].y, q[1].x, q[1].y);
      reinterpret_cast<float4*>(sy)[o4] = make_float4(q[2].x, q[2].y, q[3].x, q[3].y);
      continue;
    } else {
      const T* ex = rawx + 4 * i;
      const T* ey = rawy + 4 * i;
      a = make_float4(Ld<T>::f(ex[0]), Ld<T>::f(ex[1]), Ld<T>::f(ex[2]), Ld<T>::f(ex[3]));
      b = make_float4(Ld<T>::f(ey[0]), Ld<T>::f(ey[1]), Ld<T>::f(ey[2]), Ld<T>::f(ey[3]));
    }
    a.x -= p.shift; a.y -= p.shift; a.z -= p.shift; a.w -= p.shift;
    b.x -= p.shift; b.y -= p.shift; b.z -= p.shift; b.w -= p.shift;
    if constexpr (UV) {
      const float4 u = make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
      b = make_float4(a.x - b.x, a.y - b.y, a.z - b.z, a.w - b.w);
      a = u;
    }
    reinterpret_cast<float4*>(sx)[o4] = a;
    reinterpret_cast<float4*>(sy)[o4] = b;
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
template <int KW, int P>
__device__ __forceinline__ void stage_store(float* sx, float* sy, const float (&vx)[Geo<KW>::NE],
                                            const float (&vy)[Geo<KW>::NE]) {
  using G = Geo<KW>;
#pragma unroll
  for (int e = 0; e < G::NE; ++e) {
    const int idx = threadIdx.x + e * G::NT;
    if (idx < KW * G::SW) {
      const int r = idx / G::SW, c = idx - r * G::SW;
      sx[r * P + c] = vx[e];
      sy[r * P + c] = vy[e];
    }
  }
}

// ---------------------------------------------------------------------------
// blurs
// ---------------------------------------------------------------------------

// Tap index: with SYM the window is known to be symmetric (w[j] == w[KW-1-j],
// checked on the host), so only the first (KW+1)/2 taps are read and fewer
// registers hold them.
template <int KW, bool SYM>
__device__ __forceinline__ constexpr int tap(int j) {
  return (SYM && j > KW - 1 - j) ? KW - 1 - j : j;
}

// Transposed (adjoint) blurs correlate with the reversed window; FLIP selects
// w[KW-1-j].  For a symmetric window both orders give the same taps.
template <int KW, bool SYM, bool FLIP>
__device__ __forceinline__ constexpr int tapf(int j) {
  return tap<KW, SYM>(FLIP ? KW - 1 - j : j);
}

// Horizontal blur of the (x', y') planes: KW adjacent outputs from 2KW-1
// staged inputs; out[o].xy = sum_j w[j] * plane(o + j).
template <int KW, bool SYM = false>
__device__ __forceinline__ void hblur_xy(const SsimArgs& p, const float* __restrict__ sx,
                                         const float* __restrict__ sy, float4* __restrict__ out) {
  float2 acc[KW];
#pragma unroll
  for (int o = 0; o < KW; ++o) acc[o] = make_float2(0.f, 0.f);
#pragma unroll
  for (int q = 0; q < 2 * KW - 1; ++q) {
    const float2 v = make_float2(sx[q], sy[q]);
#pragma unroll
    for (int o = 0; o < KW; ++o) {
      const int j = q - o;
      if (j >= 0 && j < KW) acc[o] = __ffma2_rn(p.w2[tap<KW, SYM>(j)], v, acc[o]);
    }
  }
#pragma unroll
  for (int o = 0; o < KW; ++o) reinterpret_cast<float2*>(out + o)[0] = acc[o];
}

// Horizontal blur of the product planes (x'y', (x'-y')^2) -> out[o].zw.
template <int KW, bool SYM = false>
__device__ __forceinline__ void hblur_prod(const SsimArgs& p, const float* __restrict__ sx,
                                           const float* __restrict__ sy,
                                           float4* __restrict__ out) {
  float2 acc[KW];
#pragma unroll
  for (int o = 0; o < KW; ++o) acc[o] = make_float2(0.f, 0.f);
#pragma unroll
  for (int q = 0; q < 2 * KW - 1; ++q) {
    const float xv = sx[q], yv = sy[q];
    const float dv = xv - yv;
    const float2 v = make_float2(xv * yv, dv * dv);
#pragma unroll
    for (int o = 0; o < KW; ++o) {
      const int j = q - o;
      if (j >= 0 && j < KW) acc[o] = __ffma2_rn(p.w2[tap<KW, SYM>(j)], v, acc[o]);
    }
  }
#pragma unroll
  for (int o = 0; o < KW; ++o) reinterpret_cast<float2*>(out + o)[1] = acc[o];
}

// Horizontal blur of the four moment planes from shifted staged rows, in
// three passes of at most (KW+2)/3 outputs: out[o] = (blur x', blur y',
// blur x'y', blur (x'-y')^2).  Fewer live accumulators than two full-width
// passes, for the same number of shared loads.
// UV: the staged rows hold u = x' + y' and v = x' - y'; the four planes are
// then u, v, u^2, v^2 (one packed multiply per input; ssim_uv).
template <int KW, bool SYM, int O0, int NO, bool UV = false>
__device__ __forceinline__ void hblur4_part(const SsimArgs& p, const float* __restrict__ sx,
                                            const float* __restrict__ sy,
                                            float4* __restrict__ out) {
  float2 a[NO], b[NO];
#pragma unroll
  for (int o = 0; o < NO; ++o) a[o] = b[o] = make_float2(0.f, 0.f);
#pragma unroll
  for (int q = O0; q < O0 + NO + KW - 1; ++q) {
    const float xv = sx[q], yv = sy[q];
    const float2 c = make_float2(xv, yv);
    float2 v;
    if constexpr (UV) {
      v = __fmul2_rn(c, c);
    } else {
      const float dv = xv - yv;
      v = make_float2(xv * yv, dv * dv);
    }
#pragma unroll
    for (int o = 0; o < NO; ++o) {
      const int j = q - (O0 + o);
      if (j >= 0 && j < KW) {
        const float2 w = p.w2[tap<KW, SYM>(j)];
        a[o] = __ffma2_rn(w, c, a[o]);
        b[o] = __ffma2_rn(w, v, b[o]);
      }
    }
  }
#pragma unroll
  for (int o = 0; o < NO; ++o) out[O0 + o] = make_float4(a[o].x, a[o].y, b[o].x, b[o].y);
}

template <int KW, bool SYM, bool UV = false>
__device__ __forceinline__ void hblur4(const SsimArgs& p, const float* sx, const float* sy,
                                       float4* out) {
  constexpr int H = (KW + 2) / 3;
  hblur4_part<KW, SYM, 0, H, UV>(p, sx, sy, out);
  hblur4_part<KW, SYM, H, H, UV>(p, sx, sy, out);
  hblur4_part<KW, SYM, 2 * H, KW - 2 * H, UV>(p, sx, sy, out);
}

// Horizontal blur of two float components of float4 rows (backward scatter).
// HALF selects .xy (0) or .zw (1); NC = 1 blurs only the first of the pair.
template <int KW, int HALF, int NC, bool SYM = false, bool FLIP = false>
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
        if (NC == 2) acc[o] = __ffma2_rn(p.w2[tapf<KW, SYM, FLIP>(j)], v, acc[o]);
        else acc[o].x = fmaf(p.w2[tapf<KW, SYM, FLIP>(j)].x, v.x, acc[o].x);
      }
    }
  }
#pragma unroll
  for (int o = 0; o < KW; ++o) reinterpret_cast<float2*>(out + o)[HALF] = acc[o];
}

// Vertical blur over the register ring: the newest row sits in slot K, the
// output row needs slots K+1 .. K+KW (mod KW), oldest first.
template <int KW, int K, int NPL, bool SYM = false, bool FLIP = false>
__device__ __forceinline__ float4 vblur(const SsimArgs& p, const float4 (&ring)[KW]) {
  // even and odd taps accumulate separately: twice the independent chains
  float2 a0 = make_float2(0.f, 0.f), b0 = make_float2(0.f, 0.f);
  float2 a1 = make_float2(0.f, 0.f), b1 = make_float2(0.f, 0.f);
#pragma unroll
  for (int j = 0; j < KW; ++j) {
    const float4 h = ring[(K + 1 + j) % KW];
    float2& a = (j & 1) ? a1 : a0;
    float2& b = (j & 1) ? b1 : b0;
    const float2 wj = p.w2[tapf<KW, SYM, FLIP>(j)];
    a = __ffma2_rn(wj, make_float2(h.x, h.y), a);
    if (NPL == 4) b = __ffma2_rn(wj, make_float2(h.z, h.w), b);
    else b.x = fmaf(wj.x, h.z, b.x);
  }
  const float2 a = __fadd2_rn(a0, a1), b = __fadd2_rn(b0, b1);
  return make_float4(a.x, a.y, b.x, b.y);
}

// Static-slot dispatch of vblur for a loop index k that the unroller resolves.
template <int KW, int NPL, bool SYM = false, bool FLIP = false>
__device__ __forceinline__ float4 vblur_at(const SsimArgs& p, const float4 (&ring)[KW], int k) {
  switch (k) {
#define FAB_VB(KK) \
  case KK: return vblur<KW, (KK < KW ? KK : 0), NPL, SYM, FLIP>(p, ring);
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

// S and cs straight from blurred (U, V, U2, V2).  With mx + my = U + 2 shift,
// mx - my = V, P = (U + 2 shift)^2 and Q = V^2:  2 A1 = P - Q + 2 C1,
// 2 B1 = P + Q + 2 C1, 2 A2 = var_u - var_v + 2 C2, 2 B2 = var_u + var_v + 2 C2
// (the factors of 2 cancel in S = A1 A2 / (B1 B2) and cs = A2 / B2).  One
// approximate reciprocal serves both.
struct SsimCs {
  float S, cs;
};
template <bool CS>
__device__ __forceinline__ SsimCs ssim_uv(const SsimArgs& p, const float4& s) {
  const float us = s.x + 2.f * p.shift;
  const float P = us * us, Q = s.y * s.y;
  const float var_u = fmaf(-s.x, s.x, s.z);
  const float var_v = s.w - Q;
  const float t1 = fmaf(2.f, p.C1, P), t2 = fmaf(2.f, p.C2, var_u);
  const float a1 = t1 - Q, b1 = t1 + Q, a2 = t2 - var_v, b2 = t2 + var_v;
  const float inv = __fdividef(1.0f, b1 * b2);
  SsimCs r;
  r.S = a1 * a2 * inv;
  r.cs = CS ? a2 * b1 * inv : 0.f;
  return r;
}

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

// Host: a 4-D TMA map (x, row, channel, image) of a strided view, with the
// base rounded down to 16 bytes (the leading elements that adds are returned
// in *d).  Returns false when the view cannot be described (strides not
// multiples of 16 bytes, or no driver entry point); callers then stage with
// register loads.
bool make_row_map(CUtensorMap* map, const View& v, int dtype, int box_w, int* d);
// A 3-D map of 8-byte units {d0, d1, d2} with byte strides s1, s2 (multiples
// of 16) and box {b0, b1, 1}; elements outside the dims read as zero.
bool make_map_3d_u64(CUtensorMap* map, const void* base, unsigned long long d0,
                     unsigned long long d1, unsigned long long d2, unsigned long long s1,
                     unsigned long long s2, int b0, int b1);

struct SsimPlan {
  int strips, chunks, RH;
};

// Split rows into chunks (one block per strip x plane x chunk).  The cost
// model is waves x (rows per chunk + halo rows each chunk recomputes): few
// chunks waste the halo less, but must still fill every SM slot.
static inline SsimPlan plan_rows(int rows_total, int strips, int planes, int device,
                                 int blocks_per_sm, int halo) {
  const long long slots = (long long)sm_count(device) * blocks_per_sm;
  const long long per = (long long)strips * planes;
  int best_c = 1;
  double best = 1e300;
  const int cmax = rows_total < 256 ? rows_total : 256;
  for (int c = 1; c <= cmax; ++c) {
    const long long rh = (rows_total + c - 1) / c;
    const long long waves = (per * c + slots - 1) / slots;
    const double cost = (double)waves * (double)(rh + halo);
    if (cost < best * 0.999) {
      best = cost;
      best_c = c;
    }
  }
  SsimPlan pl;
  pl.strips = strips;
  pl.RH = (rows_total + best_c - 1) / best_c;
  pl.chunks = (rows_total + pl.RH - 1) / pl.RH;
  return pl;
}

// Last block of a launch that accumulates SSIM sums (the forward kernel, and
// the backward kernel in its fused forward mode): per-plane sums in a fixed
// order, then per-image and batch means.
static __device__ __noinline__ void ssim_fwd_finalize(const SsimArgs& p, int bpp) {
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

// The Gaussian taps of the reference-compatible entry points arrive as a
// device pointer (`wdev`): every thread reads them (a broadcast from L1/L2)
// into a private copy of the arguments, so no host copy of the window, and
// no synchronisation, is needed.
template <int KW>
__device__ __forceinline__ void load_device_taps(SsimArgs& q) {
#pragma unroll
  for (int j = 0; j < KW; ++j) {
    const float w = __ldg(q.wdev + j);
    q.w[j] = w;
    q.w2[j] = make_float2(w, w);
  }
}

}  // namespace fab
