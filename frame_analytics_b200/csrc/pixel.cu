// Pixel reductions on sm_100a: MSE / L1 / Charbonnier / Huber (+ PSNR).
//
// Semantics follow the reference's pixel kernels (fa_cuda.cu:252-359) and its
// finaliser (fa_cuda.cu:182-210):
//   term   MSE d^2, L1 |d|, Charbonnier sqrt(d^2 + eps^2), Huber
//          0.5*min(a,delta)^2 + delta*(a - min(a,delta)) with a = |d|
//   mean   sum / count (a divide, not a reciprocal multiply)
//   PSNR   bias - 10*log10(mean), bias = 10*log10(L^2)
// uint8 MSE and L1 are summed in 64-bit integers, so they are exact.
//
// Design (B200): one launch.  Every block streams its share of one image with
// 128-bit loads (4 in flight per operand per thread), reduces with warp
// shuffles, publishes one partial, and the last block to finish reduces all
// partials in a fixed order and writes every output.  Luma and border crop are
// folded into the loads (the reference materialises luma with torch ops,
// functional.py:267-271, and copies cropped views, backend.py:156-163).
#include "common.cuh"

namespace fab {

constexpr int PIX_THREADS = 256;
constexpr int PIX_WARPS = PIX_THREADS / 32;
constexpr int PIX_UNROLL = 4;

template <typename T, int OP>
struct PixTraits {
  // integer-exact accumulation: uint8 MSE and L1
  static constexpr bool kExact =
      (std::is_same<T, unsigned char>::value || std::is_same<T, unsigned short>::value) &&
      (OP == FA_OP_MSE || OP == FA_OP_L1);
  // uint8 Charbonnier / Huber read their term from a 256-entry table
  static constexpr bool kLut =
      std::is_same<T, unsigned char>::value && (OP == FA_OP_CHARB || OP == FA_OP_HUBER);
  using Acc = typename std::conditional<kExact, unsigned long long, double>::type;
};

template <int OP, typename F>
__device__ __forceinline__ F pix_term(F d, F p) {
  if (OP == FA_OP_MSE) return d * d;
  if (OP == FA_OP_L1) return fabs(d);
  if (OP == FA_OP_CHARB) return sqrt(d * d + p);
  const F a = fabs(d);
  const F lo = a < p ? a : p;
  return F(0.5) * lo * lo + p * (a - lo);
}

struct PixArgs {
  const char* a;
  const char* b;
  long long sn, sc, sh;     // element strides (a and b share them)
  int n, c, h, w;
  int bpi;                  // blocks per image
  int flat;                 // images are contiguous runs of c*h*w elements
  int luma;                 // rows kernel: project RGB to luma first
  double k0, k1, k2;        // luma coefficients (offset cancels in a - b)
  float pf;                 // op parameter, float
  double pd;                // op parameter, double
  double psnr_bias;
  unsigned int* counter;
  void* partial;            // [n][bpi] Acc
  double* out_per_image;
  double* out_total;
  double* out_psnr_per_image;
  double* out_psnr_total;
  unsigned long long* out_isum;
};

// ---- per-element accumulation ------------------------------------------------

// 16 bytes of each operand -> accumulator.
template <typename T, int OP>
__device__ __forceinline__ void accum_vec(const uint4& va, const uint4& vb,
                                          typename PixTraits<T, OP>::Acc& acc,
                                          const float* lut, float pf, double pd) {
  using Tr = PixTraits<T, OP>;
  if constexpr (Tr::kExact && sizeof(T) == 2) {
    // uint16: |d| < 2^16, d^2 < 2^32 per element, summed in 64 bits
    const unsigned short* ea = reinterpret_cast<const unsigned short*>(&va);
    const unsigned short* eb = reinterpret_cast<const unsigned short*>(&vb);
    unsigned long long s = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const unsigned d = ea[i] > eb[i] ? (unsigned)ea[i] - eb[i] : (unsigned)eb[i] - ea[i];
      s += (OP == FA_OP_MSE) ? (unsigned long long)(d * d) : (unsigned long long)d;
    }
    acc += s;
  } else if constexpr (Tr::kExact) {
    const unsigned wa[4] = {va.x, va.y, va.z, va.w};
    const unsigned wb[4] = {vb.x, vb.y, vb.z, vb.w};
    unsigned s = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const unsigned d = __vabsdiffu4(wa[i], wb[i]);
      s = (OP == FA_OP_MSE) ? __dp4a(d, d, s) : __dp4a(d, 0x01010101u, s);
    }
    acc += s;
  } else if constexpr (Tr::kLut) {
    const unsigned wa[4] = {va.x, va.y, va.z, va.w};
    const unsigned wb[4] = {vb.x, vb.y, vb.z, vb.w};
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const unsigned d = __vabsdiffu4(wa[i], wb[i]);
      s += lut[d & 0xff] + lut[(d >> 8) & 0xff] + lut[(d >> 16) & 0xff] + lut[d >> 24];
    }
    acc += (double)s;
  } else if constexpr (std::is_same<T, double>::value) {
    const double2 xa = *reinterpret_cast<const double2*>(&va);
    const double2 xb = *reinterpret_cast<const double2*>(&vb);
    acc += pix_term<OP, double>(xa.x - xb.x, pd) + pix_term<OP, double>(xa.y - xb.y, pd);
  } else {
    constexpr int E = 16 / sizeof(T);
    const T* ea = reinterpret_cast<const T*>(&va);
    const T* eb = reinterpret_cast<const T*>(&vb);
    if constexpr (OP == FA_OP_MSE) {
      // float term, float64 sum (fa_cuda.cu:262-281)
#pragma unroll
      for (int i = 0; i < E; ++i) {
        const float d = Ld<T>::f(ea[i]) - Ld<T>::f(eb[i]);
        acc += (double)(d * d);
      }
    } else {
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < E; ++i)
        s += pix_term<OP, float>(Ld<T>::f(ea[i]) - Ld<T>::f(eb[i]), pf);
      acc += (double)s;
    }
  }
}

template <typename T, int OP>
__device__ __forceinline__ void accum_one(T x, T y, typename PixTraits<T, OP>::Acc& acc,
                                          const float* lut, float pf, double pd) {
  using Tr = PixTraits<T, OP>;
  if constexpr (Tr::kExact) {
    const long long d = (long long)x - (long long)y;
    acc += (OP == FA_OP_MSE) ? (unsigned long long)(d * d)
                             : (unsigned long long)(d < 0 ? -d : d);
  } else if constexpr (Tr::kLut) {
    const int d = (int)x - (int)y;
    acc += (double)lut[d < 0 ? -d : d];
  } else if constexpr (std::is_same<T, double>::value) {
    acc += pix_term<OP, double>(x - y, pd);
  } else {
    const float d = Ld<T>::f(x) - Ld<T>::f(y);
    if (OP == FA_OP_MSE) acc += (double)(d * d);
    else acc += (double)pix_term<OP, float>(d, pf);
  }
}

// Reduce a run of `len` elements starting at pa / pb.  The caller's lanes
// (`lane` of `nl`) cooperate; 16-byte vectors when both pointers share their
// alignment, scalar otherwise.
template <typename T, int OP>
__device__ __forceinline__ void reduce_run(const T* pa, const T* pb, long long len,
                                           long long lane, long long nl,
                                           typename PixTraits<T, OP>::Acc& acc,
                                           const float* lut, float pf, double pd) {
  constexpr int E = 16 / sizeof(T);
  const uintptr_t ua = reinterpret_cast<uintptr_t>(pa);
  const uintptr_t ub = reinterpret_cast<uintptr_t>(pb);
  if (((ua ^ ub) & 15u) != 0) {
    for (long long i = lane; i < len; i += nl) accum_one<T, OP>(ldro(pa + i), ldro(pb + i), acc, lut, pf, pd);
    return;
  }
  long long head = (long long)(((16u - (ua & 15u)) & 15u) / sizeof(T));
  if (head > len) head = len;
  const long long nv = (len - head) / E;
  const long long tail0 = head + nv * E;
  if (lane < head) accum_one<T, OP>(ldro(pa + lane), ldro(pb + lane), acc, lut, pf, pd);
  const long long t = tail0 + lane;
  if (t < len) {
    // tail is < E elements; lanes beyond E do nothing here
    for (long long i = t; i < len; i += nl) accum_one<T, OP>(ldro(pa + i), ldro(pb + i), acc, lut, pf, pd);
  }
  const uint4* va = reinterpret_cast<const uint4*>(pa + head);
  const uint4* vb = reinterpret_cast<const uint4*>(pb + head);
  long long v = lane;
  for (; v + (PIX_UNROLL - 1) * nl < nv; v += PIX_UNROLL * nl) {
    uint4 xa[PIX_UNROLL], xb[PIX_UNROLL];
#pragma unroll
    for (int u = 0; u < PIX_UNROLL; ++u) {
      xa[u] = __ldg(va + v + u * nl);
      xb[u] = __ldg(vb + v + u * nl);
    }
#pragma unroll
    for (int u = 0; u < PIX_UNROLL; ++u) accum_vec<T, OP>(xa[u], xb[u], acc, lut, pf, pd);
  }
  if (v < nv) {
    // the remainder: every load issued before any is used
    uint4 xa[PIX_UNROLL], xb[PIX_UNROLL];
#pragma unroll
    for (int u = 0; u < PIX_UNROLL; ++u) {
      const bool ok = v + u * nl < nv;
      xa[u] = ok ? __ldg(va + v + u * nl) : make_uint4(0, 0, 0, 0);
      xb[u] = ok ? __ldg(vb + v + u * nl) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < PIX_UNROLL; ++u)
      if (v + u * nl < nv) accum_vec<T, OP>(xa[u], xb[u], acc, lut, pf, pd);
  }
}

// reduce_run for the contiguous-image kernel, with one contiguous span of the
// run's 16-byte vectors per block (block `blk` of `nblk`, thread `t` of
// PIX_THREADS): every step reads PIX_UNROLL x 4 KB of each operand as one
// coalesced sweep, and each block streams its own DRAM pages instead of
// striding the whole image.  Block 0 also takes the unaligned head and tail.
template <typename T, int OP>
__device__ __forceinline__ void reduce_span(const T* pa, const T* pb, long long len, int blk,
                                            int nblk, int t,
                                            typename PixTraits<T, OP>::Acc& acc,
                                            const float* lut, float pf, double pd) {
  constexpr int E = 16 / sizeof(T);
  constexpr int STEP = PIX_UNROLL * PIX_THREADS;
  const uintptr_t ua = reinterpret_cast<uintptr_t>(pa);
  const uintptr_t ub = reinterpret_cast<uintptr_t>(pb);
  if (((ua ^ ub) & 15u) != 0) {
    reduce_run<T, OP>(pa, pb, len, (long long)blk * PIX_THREADS + t,
                      (long long)nblk * PIX_THREADS, acc, lut, pf, pd);
    return;
  }
  long long head = (long long)(((16u - (ua & 15u)) & 15u) / sizeof(T));
  if (head > len) head = len;
  const long long nv = (len - head) / E;
  const long long tail0 = head + nv * E;
  if (blk == 0) {
    if (t < head) accum_one<T, OP>(ldro(pa + t), ldro(pb + t), acc, lut, pf, pd);
    if (tail0 + t < len) accum_one<T, OP>(ldro(pa + tail0 + t), ldro(pb + tail0 + t), acc, lut, pf, pd);
  }
  // spans are whole steps, so only the last block's last step is ragged
  const long long per = (nv + (long long)nblk * STEP - 1) / ((long long)nblk * STEP) * STEP;
  const long long lo = (long long)blk * per;
  const long long hi = lo + per < nv ? lo + per : nv;
  const uint4* va = reinterpret_cast<const uint4*>(pa + head);
  const uint4* vb = reinterpret_cast<const uint4*>(pb + head);
  for (long long v0 = lo; v0 < hi; v0 += STEP) {
    uint4 xa[PIX_UNROLL], xb[PIX_UNROLL];
    if (v0 + STEP <= hi) {
#pragma unroll
      for (int u = 0; u < PIX_UNROLL; ++u) {
        xa[u] = __ldg(va + v0 + u * PIX_THREADS + t);
        xb[u] = __ldg(vb + v0 + u * PIX_THREADS + t);
      }
#pragma unroll
      for (int u = 0; u < PIX_UNROLL; ++u) accum_vec<T, OP>(xa[u], xb[u], acc, lut, pf, pd);
    } else {
#pragma unroll
      for (int u = 0; u < PIX_UNROLL; ++u) {
        const long long v = v0 + u * PIX_THREADS + t;
        xa[u] = v < hi ? __ldg(va + v) : make_uint4(0, 0, 0, 0);
        xb[u] = v < hi ? __ldg(vb + v) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < PIX_UNROLL; ++u)
        if (v0 + u * PIX_THREADS + t < hi) accum_vec<T, OP>(xa[u], xb[u], acc, lut, pf, pd);
    }
  }
}

// Luma rows: dY = k0*dR + k1*dG + k2*dB in float64 (the luma offset cancels).
template <typename T, int OP>
__device__ __forceinline__ void reduce_luma_row(const T* ra, const T* rb, long long sc,
                                                int len, int lane, double& acc,
                                                double k0, double k1, double k2, double pd) {
  for (int i = lane; i < len; i += 32) {
    const double dr = Ld<T>::d(ldro(ra + i)) - Ld<T>::d(ldro(rb + i));
    const double dg = Ld<T>::d(ldro(ra + sc + i)) - Ld<T>::d(ldro(rb + sc + i));
    const double db = Ld<T>::d(ldro(ra + 2 * sc + i)) - Ld<T>::d(ldro(rb + 2 * sc + i));
    const double d = fma(k0, dr, fma(k1, dg, k2 * db));
    acc += pix_term<OP, double>(d, pd);
  }
}

// uint8 luma rows, 16 pixels per lane step when the six row pointers agree
// on alignment.
template <int OP>
__device__ __forceinline__ void reduce_luma_row_u8(const unsigned char* ra,
                                                   const unsigned char* rb, long long sc,
                                                   int len, int lane, double& acc,
                                                   double k0, double k1, double k2,
                                                   double pd) {
  const uintptr_t u0 = reinterpret_cast<uintptr_t>(ra) & 15u;
  const bool same = ((reinterpret_cast<uintptr_t>(rb) & 15u) == u0) &&
                    ((reinterpret_cast<uintptr_t>(ra + sc) & 15u) == u0) &&
                    ((reinterpret_cast<uintptr_t>(rb + sc) & 15u) == u0);
  if (!same) {
    reduce_luma_row<unsigned char, OP>(ra, rb, sc, len, lane, acc, k0, k1, k2, pd);
    return;
  }
  int head = (int)((16u - u0) & 15u);
  if (head > len) head = len;
  const int nv = (len - head) >> 4;
  const int tail0 = head + (nv << 4);
  auto px = [&](int i) {
    const double dr = (double)((int)ra[i] - (int)rb[i]);
    const double dg = (double)((int)ra[sc + i] - (int)rb[sc + i]);
    const double db = (double)((int)ra[2 * sc + i] - (int)rb[2 * sc + i]);
    const double d = fma(k0, dr, fma(k1, dg, k2 * db));
    acc += pix_term<OP, double>(d, pd);
  };
  if (lane < head) px(lane);
  if (tail0 + lane < len) px(tail0 + lane);
  for (int v = lane; v < nv; v += 32) {
    const int o = head + (v << 4);
    const uint4 A0 = __ldg(reinterpret_cast<const uint4*>(ra + o));
    const uint4 B0 = __ldg(reinterpret_cast<const uint4*>(rb + o));
    const uint4 A1 = __ldg(reinterpret_cast<const uint4*>(ra + sc + o));
    const uint4 B1 = __ldg(reinterpret_cast<const uint4*>(rb + sc + o));
    const uint4 A2 = __ldg(reinterpret_cast<const uint4*>(ra + 2 * sc + o));
    const uint4 B2 = __ldg(reinterpret_cast<const uint4*>(rb + 2 * sc + o));
    const unsigned char* a0 = reinterpret_cast<const unsigned char*>(&A0);
    const unsigned char* b0 = reinterpret_cast<const unsigned char*>(&B0);
    const unsigned char* a1 = reinterpret_cast<const unsigned char*>(&A1);
    const unsigned char* b1 = reinterpret_cast<const unsigned char*>(&B1);
    const unsigned char* a2 = reinterpret_cast<const unsigned char*>(&A2);
    const unsigned char* b2 = reinterpret_cast<const unsigned char*>(&B2);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const double d = fma(k0, (double)((int)a0[j] - (int)b0[j]),
                           fma(k1, (double)((int)a1[j] - (int)b1[j]),
                               k2 * (double)((int)a2[j] - (int)b2[j])));
      acc += pix_term<OP, double>(d, pd);
    }
  }
}

template <typename T, int OP>
__device__ __forceinline__ void fill_lut(float* lut, float pf) {
  if constexpr (PixTraits<T, OP>::kLut) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x)
      lut[i] = pix_term<OP, float>((float)i, pf);
    __syncthreads();
  }
}

// Last-block finaliser: per-image sums in a fixed order, then means, PSNR,
// exact sums and the batch total.
template <typename Acc>
__device__ void pix_finalize(const PixArgs& p, double n_per_image) {
  __shared__ Acc s_red[32];
  __shared__ Acc s_img[64];  // per-image sums of small batches stay on chip
  Acc* part = static_cast<Acc*>(p.partial);
  const bool on_chip = p.n <= 64;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  // 1. per-image sums, one warp per image; kept in shared memory (small
  //    batches) or in slot 0 of the image's partials row
  for (int img = wid; img < p.n; img += PIX_WARPS) {
    Acc s = 0;
    for (int i = lane; i < p.bpi; i += 32) s += part[(long long)img * p.bpi + i];
    s = warp_sum(s);
    if (lane == 0) {
      if (on_chip) s_img[img] = s;
      else part[(long long)img * p.bpi] = s;
      const double v = (double)s / n_per_image;
      if (p.out_per_image) p.out_per_image[img] = v;
      if (p.psnr_bias != FA_PSNR_NONE && p.out_psnr_per_image)
        p.out_psnr_per_image[img] = p.psnr_bias - 10.0 * log10(v);
      if (p.out_isum) p.out_isum[img] = (unsigned long long)s;
    }
  }
  __syncthreads();
  if (!on_chip) __threadfence_block();
  // 2. batch total over the per-image sums, fixed order
  Acc t = 0;
  for (int img = threadIdx.x; img < p.n; img += blockDim.x)
    t += on_chip ? s_img[img] : part[(long long)img * p.bpi];
  t = block_sum(t, s_red);
  if (threadIdx.x == 0) {
    const double v = (double)t / (n_per_image * (double)p.n);
    if (p.out_total) *p.out_total = v;
    if (p.psnr_bias != FA_PSNR_NONE && p.out_psnr_total)
      *p.out_psnr_total = p.psnr_bias - 10.0 * log10(v);
  }
}

// Contiguous images: block (bx, img) streams span bx of image img's c*h*w
// elements.
template <typename T, int OP>
__global__ void __launch_bounds__(PIX_THREADS, 6) pixel_flat_kernel(PixArgs p) {
  using Tr = PixTraits<T, OP>;
  using Acc = typename Tr::Acc;
  __shared__ float s_lut[Tr::kLut ? 256 : 1];
  __shared__ Acc s_red[32];
  __shared__ int s_flag;
  fill_lut<T, OP>(s_lut, p.pf);

  const int img = blockIdx.y;
  const long long per = (long long)p.c * p.h * p.w;
  const T* pa = reinterpret_cast<const T*>(p.a) + (long long)img * p.sn;
  const T* pb = reinterpret_cast<const T*>(p.b) + (long long)img * p.sn;
  Acc acc = 0;
  reduce_span<T, OP>(pa, pb, per, blockIdx.x, p.bpi, threadIdx.x, acc, s_lut, p.pf, p.pd);
  acc = block_sum(acc, s_red);
  if (threadIdx.x == 0) static_cast<Acc*>(p.partial)[(long long)img * p.bpi + blockIdx.x] = acc;
  if (last_block_arrived(p.counter, gridDim.x * gridDim.y, &s_flag))
    pix_finalize<Acc>(p, (double)per);
}

// Strided rows (border crop, arbitrary strides) and luma: one warp per row.
template <typename T, int OP, bool LUMA>
__global__ void __launch_bounds__(PIX_THREADS) pixel_rows_kernel(PixArgs p) {
  using Tr = PixTraits<T, OP>;
  using Acc = typename std::conditional<LUMA, double, typename Tr::Acc>::type;
  __shared__ float s_lut[(!LUMA && Tr::kLut) ? 256 : 1];
  __shared__ Acc s_red[32];
  __shared__ int s_flag;
  if constexpr (!LUMA) fill_lut<T, OP>(s_lut, p.pf);

  const int img = blockIdx.y;
  const int lane = threadIdx.x & 31;
  const int rows = LUMA ? p.h : p.c * p.h;
  const int gw = blockIdx.x * PIX_WARPS + (threadIdx.x >> 5);
  const int nw = p.bpi * PIX_WARPS;
  Acc acc = 0;
  for (int r = gw; r < rows; r += nw) {
    const int ch = LUMA ? 0 : r / p.h;
    const int hh = LUMA ? r : r - ch * p.h;
    const long long off = (long long)img * p.sn + (long long)ch * p.sc + (long long)hh * p.sh;
    const T* ra = reinterpret_cast<const T*>(p.a) + off;
    const T* rb = reinterpret_cast<const T*>(p.b) + off;
    if constexpr (LUMA) {
      if constexpr (std::is_same<T, unsigned char>::value)
        reduce_luma_row_u8<OP>(ra, rb, p.sc, p.w, lane, acc, p.k0, p.k1, p.k2, p.pd);
      else
        reduce_luma_row<T, OP>(ra, rb, p.sc, p.w, lane, acc, p.k0, p.k1, p.k2, p.pd);
    } else {
      typename Tr::Acc a2 = 0;
      reduce_run<T, OP>(ra, rb, p.w, lane, 32, a2, s_lut, p.pf, p.pd);
      acc += (Acc)a2;
    }
  }
  acc = block_sum(acc, s_red);
  if (threadIdx.x == 0) static_cast<Acc*>(p.partial)[(long long)img * p.bpi + blockIdx.x] = acc;
  if (last_block_arrived(p.counter, gridDim.x * gridDim.y, &s_flag))
    pix_finalize<Acc>(p, (double)(LUMA ? 1 : p.c) * p.h * p.w);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

static int pix_bpi(int n_images, int device) {
  // ~8 resident 256-thread blocks per SM, split evenly over the images
  const int sms = sm_count(device);
  long long bpi = ((long long)sms * 8 + n_images - 1) / n_images;
  if (bpi < 1) bpi = 1;
  if (bpi > 4096) bpi = 4096;
  return (int)bpi;
}

// Blocks per image so that the whole grid is one wave of resident blocks
// (never more than the workspace was sized for).
template <auto KERN>
static int wave_bpi(const PixArgs& p, int device) {
  static int occ[64] = {0};  // one cache per kernel instantiation
  auto* kern = KERN;
  int nb = 0;
  if (device >= 0 && device < 64 && occ[device] > 0) {
    nb = occ[device];
  } else {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, PIX_THREADS, 0) != cudaSuccess ||
        nb <= 0)
      nb = 4;
    if (device >= 0 && device < 64) occ[device] = nb;
  }
  long long bpi = (long long)nb * sm_count(device) / p.n;
  if (bpi < 1) bpi = 1;
  return bpi < p.bpi ? (int)bpi : p.bpi;
}

template <typename T>
static int launch_pixel_t(PixArgs& p, int op, int device, cudaStream_t st) {
#define FAB_PIX_OP(OPV)                                                                  \
  if (p.luma) {                                                                          \
    p.bpi = wave_bpi<pixel_rows_kernel<T, OPV, true>>(p, device);                        \
    pixel_rows_kernel<T, OPV, true><<<dim3(p.bpi, p.n), PIX_THREADS, 0, st>>>(p);        \
  } else if (p.flat) {                                                                   \
    p.bpi = wave_bpi<pixel_flat_kernel<T, OPV>>(p, device);                              \
    pixel_flat_kernel<T, OPV><<<dim3(p.bpi, p.n), PIX_THREADS, 0, st>>>(p);              \
  } else {                                                                               \
    p.bpi = wave_bpi<pixel_rows_kernel<T, OPV, false>>(p, device);                       \
    pixel_rows_kernel<T, OPV, false><<<dim3(p.bpi, p.n), PIX_THREADS, 0, st>>>(p);       \
  }
  switch (op) {
    case FA_OP_MSE: FAB_PIX_OP(FA_OP_MSE); break;
    case FA_OP_L1: FAB_PIX_OP(FA_OP_L1); break;
    case FA_OP_CHARB: FAB_PIX_OP(FA_OP_CHARB); break;
    case FA_OP_HUBER: FAB_PIX_OP(FA_OP_HUBER); break;
    default: return FA_E_OP;
  }
#undef FAB_PIX_OP
  FAB_LAUNCH_CHECK();
  return FA_OK;
}

int pixel_reduce_impl(const View& a, const View& b, int dtype, const double* luma,
                      int op, double param, double psnr_bias, void* ws, size_t ws_bytes,
                      double* out_pi, double* out_tot, double* out_ppi, double* out_ptot,
                      unsigned long long* out_isum, int device, cudaStream_t st) {
  if (!a.data || !b.data || !ws) return FA_E_ARG;
  if (op < 0 || op > 3) return FA_E_OP;
  if (a.n <= 0 || a.c <= 0 || a.h <= 0 || a.w <= 0) return FA_E_SHAPE;
  if (a.n != b.n || a.c != b.c || a.h != b.h || a.w != b.w) return FA_E_SHAPE;
  if (a.sn != b.sn || a.sc != b.sc || a.sh != b.sh) return FA_E_SHAPE;
  if (luma && a.c != 3) return FA_E_SHAPE;
  PixArgs p{};
  p.a = static_cast<const char*>(a.data);
  p.b = static_cast<const char*>(b.data);
  p.sn = a.sn; p.sc = a.sc; p.sh = a.sh;
  p.n = a.n; p.c = a.c; p.h = a.h; p.w = a.w;
  p.bpi = pix_bpi(a.n, device);
  p.flat = (!luma && a.sh == a.w && a.sc == (long long)a.h * a.w) ? 1 : 0;
  p.luma = luma ? 1 : 0;
  if (luma) { p.k0 = luma[0]; p.k1 = luma[1]; p.k2 = luma[2]; }
  p.pf = (float)param;
  p.pd = param;
  p.psnr_bias = psnr_bias;
  const size_t need = FAB_COUNTER_BYTES + (size_t)a.n * p.bpi * 8;
  if (ws_bytes < need) return FA_E_ARG;
  p.counter = static_cast<unsigned int*>(ws);
  p.partial = static_cast<char*>(ws) + FAB_COUNTER_BYTES;
  p.out_per_image = out_pi; p.out_total = out_tot;
  p.out_psnr_per_image = out_ppi; p.out_psnr_total = out_ptot;
  p.out_isum = out_isum;
  switch (dtype) {
    case FA_U8: return launch_pixel_t<unsigned char>(p, op, device, st);
    case FA_F16: return launch_pixel_t<f16_t>(p, op, device, st);
    case FA_BF16: return launch_pixel_t<bf16_t>(p, op, device, st);
    case FA_F32: return launch_pixel_t<float>(p, op, device, st);
    case FA_F64: return launch_pixel_t<double>(p, op, device, st);
    case FA_U16: return launch_pixel_t<unsigned short>(p, op, device, st);
    default: return FA_E_DTYPE;
  }
}

size_t pixel_ws_bytes(int n_images, int device) {
  return FAB_COUNTER_BYTES + (size_t)n_images * pix_bpi(n_images, device) * 8;
}

}  // namespace fab

// ---------------------------------------------------------------------------
// backward of the pixel reductions (autograd through mse / l1 / charbonnier /
// huber used as training losses; the reference falls back to torch autograd
// for these, functional.py:1097-1141).  Elementwise: dL/dx = s * t'(d),
// dL/dy = -dL/dx, s = upstream / count.  With luma the derivative of the luma
// difference is spread over R, G, B by its coefficients.
// ---------------------------------------------------------------------------
namespace fab {

template <int OP>
__device__ __forceinline__ float pix_dterm(float d, float p) {
  if (OP == FA_OP_MSE) return 2.f * d;
  if (OP == FA_OP_L1) return d > 0.f ? 1.f : (d < 0.f ? -1.f : 0.f);
  if (OP == FA_OP_CHARB) return d / sqrtf(d * d + p);
  const float a = fabsf(d);
  return a <= p ? d : (d > 0.f ? p : -p);
}

struct PixBwdArgs {
  const float* x;
  const float* y;
  int N, C, H, W;
  float k0, k1, k2;
  float pf;
  const double* g;
  int per_image;
  double count;   // elements behind one output value
  float* dx;
  float* dy;
};

template <int OP, bool LUMA>
__global__ void __launch_bounds__(256) pixel_bwd_kernel(PixBwdArgs p) {
  const long long hw = (long long)p.H * p.W;
  const long long per = LUMA ? hw : (long long)p.C * hw;   // work items per image
  const long long total = per * p.N;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long n = i / per;
    const float s = (float)(__ldg(p.g + (p.per_image ? n : 0)) / p.count);
    if constexpr (LUMA) {
      const long long o = n * 3 * hw + (i - n * per);
      const float d = p.k0 * (__ldg(p.x + o) - __ldg(p.y + o)) +
                      p.k1 * (__ldg(p.x + o + hw) - __ldg(p.y + o + hw)) +
                      p.k2 * (__ldg(p.x + o + 2 * hw) - __ldg(p.y + o + 2 * hw));
      const float t = s * pix_dterm<OP>(d, p.pf);
      if (p.dx) { p.dx[o] = p.k0 * t; p.dx[o + hw] = p.k1 * t; p.dx[o + 2 * hw] = p.k2 * t; }
      if (p.dy) { p.dy[o] = -p.k0 * t; p.dy[o + hw] = -p.k1 * t; p.dy[o + 2 * hw] = -p.k2 * t; }
    } else {
      const float t = s * pix_dterm<OP>(__ldg(p.x + i) - __ldg(p.y + i), p.pf);
      if (p.dx) p.dx[i] = t;
      if (p.dy) p.dy[i] = -t;
    }
  }
}

// ---------------------------------------------------------------------------
// A pixel loss and its gradient in one read (training with mse / l1 /
// charbonnier / huber as the loss): contiguous float32 [N, per] only.  Each
// thread sums its penalties as the forward does (float term, float64 sum) and
// writes dL/dx = norm * t'(d) (and dL/dy = -dL/dx) for an upstream gradient
// of 1; norm = 1 / count of the value the gradient is of (the batch mean, or
// each image's mean).  Block partials and the last-block finaliser are those
// of the pixel reductions.
// ---------------------------------------------------------------------------
template <int OP, bool VEC>
__global__ void __launch_bounds__(PIX_THREADS, 4) pixel_loss_grad_kernel(PixArgs p, float norm,
                                                                        float* dx, float* dy) {
  __shared__ double s_red[32];
  __shared__ int s_flag;
  const int img = blockIdx.y;
  const long long per = (long long)p.c * p.h * p.w;
  const float* xa = reinterpret_cast<const float*>(p.a) + (long long)img * per;
  const float* ya = reinterpret_cast<const float*>(p.b) + (long long)img * per;
  float* gx = dx ? dx + (long long)img * per : nullptr;
  float* gy = dy ? dy + (long long)img * per : nullptr;
  const long long t0 = (long long)blockIdx.x * PIX_THREADS + threadIdx.x;
  const long long step = (long long)p.bpi * PIX_THREADS;
  double acc = 0.0;
  auto one = [&](float d, float& g) {
    if (OP == FA_OP_MSE) acc += (double)(d * d);
    else acc += (double)pix_term<OP, float>(d, p.pf);
    g = norm * pix_dterm<OP>(d, p.pf);
  };
  if constexpr (VEC) {
    const long long n4 = per >> 2;
    for (long long v = t0; v < n4; v += step) {
      const float4 a = __ldcs(reinterpret_cast<const float4*>(xa) + v);
      const float4 b = __ldcs(reinterpret_cast<const float4*>(ya) + v);
      float4 g;
      one(a.x - b.x, g.x);
      one(a.y - b.y, g.y);
      one(a.z - b.z, g.z);
      one(a.w - b.w, g.w);
      if (gx) __stcs(reinterpret_cast<float4*>(gx) + v, g);
      if (gy) __stcs(reinterpret_cast<float4*>(gy) + v, make_float4(-g.x, -g.y, -g.z, -g.w));
    }
  } else {
    for (long long i = t0; i < per; i += step) {
      float g;
      one(__ldg(xa + i) - __ldg(ya + i), g);
      if (gx) gx[i] = g;
      if (gy) gy[i] = -g;
    }
  }
  acc = block_sum(acc, s_red);
  if (threadIdx.x == 0) static_cast<double*>(p.partial)[(long long)img * p.bpi + blockIdx.x] = acc;
  if (last_block_arrived(p.counter, gridDim.x * gridDim.y, &s_flag))
    pix_finalize<double>(p, (double)per);
}

int pixel_loss_grad_impl(const float* x, const float* y, int N, long long per, int op,
                         double param, int per_image, void* ws, size_t ws_bytes,
                         double* out_per_image, double* out_total, float* dx, float* dy,
                         int device, cudaStream_t st) {
  if (!x || !y || !ws || (!dx && !dy)) return FA_E_ARG;
  if (N <= 0 || per <= 0) return FA_E_SHAPE;
  if (op < 0 || op > 3) return FA_E_OP;
  PixArgs p{};
  p.a = reinterpret_cast<const char*>(x);
  p.b = reinterpret_cast<const char*>(y);
  p.n = N; p.c = 1; p.h = 1; p.w = (int)per;
  if ((long long)p.w != per) return FA_E_SHAPE;
  p.sn = per; p.sc = per; p.sh = per;
  p.flat = 1;
  p.pf = (float)param;
  p.pd = param;
  p.psnr_bias = FA_PSNR_NONE;
  p.bpi = pix_bpi(N, device);
  const size_t need = FAB_COUNTER_BYTES + (size_t)N * p.bpi * 8;
  if (ws_bytes < need) return FA_E_ARG;
  p.counter = static_cast<unsigned int*>(ws);
  p.partial = static_cast<char*>(ws) + FAB_COUNTER_BYTES;
  p.out_per_image = out_per_image;
  p.out_total = out_total;
  const float norm = (float)(1.0 / (per_image ? (double)per : (double)per * N));
  const bool vec = per % 4 == 0 &&
                   ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y) |
                     reinterpret_cast<uintptr_t>(dx) | reinterpret_cast<uintptr_t>(dy)) & 15u) == 0;
#define FAB_PLG(OPV)                                                                        \
  if (vec) {                                                                                \
    p.bpi = wave_bpi<pixel_loss_grad_kernel<OPV, true>>(p, device);                         \
    pixel_loss_grad_kernel<OPV, true><<<dim3(p.bpi, N), PIX_THREADS, 0, st>>>(p, norm, dx, dy); \
  } else {                                                                                  \
    p.bpi = wave_bpi<pixel_loss_grad_kernel<OPV, false>>(p, device);                        \
    pixel_loss_grad_kernel<OPV, false><<<dim3(p.bpi, N), PIX_THREADS, 0, st>>>(p, norm, dx, dy); \
  }
  switch (op) {
    case FA_OP_MSE: FAB_PLG(FA_OP_MSE); break;
    case FA_OP_L1: FAB_PLG(FA_OP_L1); break;
    case FA_OP_CHARB: FAB_PLG(FA_OP_CHARB); break;
    default: FAB_PLG(FA_OP_HUBER); break;
  }
#undef FAB_PLG
  FAB_LAUNCH_CHECK();
  return FA_OK;
}

int pixel_backward_impl(const float* x, const float* y, int N, int C, int H, int W,
                        const double* luma, int op, double param, const double* g,
                        int per_image, float* dx, float* dy, int device, cudaStream_t st) {
  if (!x || !y || !g || (!dx && !dy)) return FA_E_ARG;
  if (N <= 0 || C <= 0 || H <= 0 || W <= 0) return FA_E_SHAPE;
  if (luma && C != 3) return FA_E_SHAPE;
  if (op < 0 || op > 3) return FA_E_OP;
  PixBwdArgs p{};
  p.x = x; p.y = y; p.N = N; p.C = C; p.H = H; p.W = W;
  if (luma) { p.k0 = (float)luma[0]; p.k1 = (float)luma[1]; p.k2 = (float)luma[2]; }
  p.pf = (float)param;
  p.g = g;
  p.per_image = per_image;
  const double per = (double)(luma ? 1 : C) * H * W;
  p.count = per_image ? per : per * N;
  p.dx = dx; p.dy = dy;
  const long long work = (long long)N * (luma ? 1 : C) * H * W;
  long long blocks = (work + 255) / 256;
  const long long cap = (long long)sm_count(device) * 8;
  if (blocks > cap) blocks = cap;
#define FAB_PB(OPV)                                                                   \
  if (luma) pixel_bwd_kernel<OPV, true><<<(unsigned)blocks, 256, 0, st>>>(p);          \
  else pixel_bwd_kernel<OPV, false><<<(unsigned)blocks, 256, 0, st>>>(p);
  switch (op) {
    case FA_OP_MSE: FAB_PB(FA_OP_MSE); break;
    case FA_OP_L1: FAB_PB(FA_OP_L1); break;
    case FA_OP_CHARB: FAB_PB(FA_OP_CHARB); break;
    default: FAB_PB(FA_OP_HUBER); break;
  }
#undef FAB_PB
  FAB_LAUNCH_CHECK();
  return FA_OK;
}

}  // namespace fab

// ---------------------------------------------------------------------------
// Pixel reduction without caller-provided scratch.
//
// Some callers cannot allocate device memory at all: a plugin that only ever
// sees the host application's frame buffers, code running where cudaMalloc is
// forbidden or unavailable, or a caller whose allocator is owned by someone
// else.  They still need the reduction's scratch (grid-completion counters and
// per-block partial sums).  This variant keeps that scratch in one fixed
// array in device global memory that is part of the library image: every GPU
// that loads the library holds these bytes until the process exits, and no
// call allocates anything.
//
//   * Limit: FA_B200_NOALLOC_SCRATCH_BYTES of scratch, which covers batches of
//     up to FA_B200_NOALLOC_MAX_IMAGES images; larger batches are rejected
//     with FA_E_SHAPE before anything is launched.
//   * The array is shared by every call on a device and keeps the last call's
//     contents.  Each call clears the counters it needs on its own stream
//     first.  Calls that may run at the same time on the GPU (different
//     streams, several host threads) race on the array and give wrong results;
//     serialise them.
//   * The first call on each device looks the array's device address up
//     (cudaGetSymbolAddress, with that device current) and caches it; make
//     that first call before any stream capture.
// ---------------------------------------------------------------------------
#include <cuda.h>

#include <mutex>

namespace fab {

static __device__ __align__(256) unsigned char g_noalloc_scratch[FA_B200_NOALLOC_SCRATCH_BYTES];

// Device address of g_noalloc_scratch in the current context of `device`.
// In host code the symbol itself is only a host-side stand-in, never a
// device pointer, so the address must come from the runtime.  It is looked
// up once per (device, context): a context created anew (after
// cudaDeviceReset, or another context made current) gets its own lookup
// instead of a stale address.
typedef CUresult (*CtxGetCurrentFn)(CUcontext*);

static CUcontext current_context() {
  static CtxGetCurrentFn fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<CtxGetCurrentFn>(nullptr);
    return reinterpret_cast<CtxGetCurrentFn>(f);
  }();
  CUcontext c = nullptr;
  if (fn) fn(&c);
  return c;
}

static int noalloc_scratch(int device, void** out) {
  constexpr int MAXD = 64;
  static std::mutex mu;
  static void* addr[MAXD] = {nullptr};
  static CUcontext ctx[MAXD] = {nullptr};
  if (device < 0 || device >= MAXD) return FA_E_ARG;
  const CUcontext cur = current_context();  // the device is current here
  std::lock_guard<std::mutex> g(mu);
  if (!addr[device] || ctx[device] != cur) {
    void* p = nullptr;
    FAB_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    addr[device] = p;
    ctx[device] = cur;
  }
  *out = addr[device];
  return FA_OK;
}

}  // namespace fab

extern "C" FA_B200_API int fa_b200_pixel_reduce_noalloc(
    const fa_view* a, const fa_view* b, const double* luma, int op, double param,
    double psnr_bias, double* out_per_image, double* out_total, double* out_psnr_per_image,
    double* out_psnr_total, uint64_t* out_isum_per_image, int device, void* stream) {
  FAB_PENDING();
  using namespace fab;
  if (!a || !b || !a->data || !b->data) return FA_E_ARG;
  if (a->dtype != b->dtype) return FA_E_DTYPE;
  if (a->n <= 0 || a->c <= 0 || a->h <= 0 || a->w <= 0) return FA_E_SHAPE;
  if (a->n > FA_B200_NOALLOC_MAX_IMAGES) return FA_E_SHAPE;
  FAB_DEVICE_SCOPE(device);
  int dev = device;
  if (dev < 0) FAB_TRY(cudaGetDevice(&dev));
  const size_t need = pixel_ws_bytes(a->n, dev);
  if (need > FA_B200_NOALLOC_SCRATCH_BYTES) return FA_E_SHAPE;
  void* ws = nullptr;
  const int rc = noalloc_scratch(dev, &ws);
  if (rc != FA_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // counters must start at zero; a previous call may have been interrupted
  FAB_TRY(cudaMemsetAsync(ws, 0, FAB_COUNTER_BYTES, st));
  return pixel_reduce_impl(to_view(*a), to_view(*b), a->dtype, luma, op, param, psnr_bias, ws,
                           FA_B200_NOALLOC_SCRATCH_BYTES, out_per_image, out_total,
                           out_psnr_per_image, out_psnr_total,
                           reinterpret_cast<unsigned long long*>(out_isum_per_image), dev, st);
}
