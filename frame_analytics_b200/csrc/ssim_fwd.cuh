// SSIM forward kernel on sm_100a (device code and launch helper; the host
// entry is ssim_fwd.cu): per-plane SSIM and cs means, the SSIM map, per
// image and batch means -- one launch.  Replaces the reference's
// ssim_fused_kernel REDUCE/MAP/CS modes + finalize (fa_cuda.cu:389-637,
// 182-234, host 1167-1283).  Layout notes: ssim_common.cuh.
#pragma once

#include <type_traits>

#include "ssim_common.cuh"

namespace fab {

// Squared-difference accumulator: exact for uint8, double otherwise (float
// terms for f16/bf16/f32 as the pixel reductions form them, double for f64).
template <typename T>
using SqAcc = typename std::conditional<std::is_same<T, unsigned char>::value ||
                                            std::is_same<T, unsigned short>::value,
                                        unsigned long long, double>::type;

// stage_convert plus the squared differences of the staged elements this
// block owns: global rows [rlo, rhi) and columns [clo, chi).  Element (r, i)
// of the staged rows is global row grow0 + r, column gcol0 + i.  Rows and
// columns outside the image arrive as zeros in both inputs and add nothing.
template <typename T, int KW, bool UV>
__device__ __forceinline__ void stage_convert_sq(const SsimArgs& p, const T* rawx, const T* rawy,
                                                 float* sx, float* sy, int grow0, int gcol0,
                                                 int rlo, int rhi, int clo, int chi,
                                                 SqAcc<T>& acc) {
  using R = Raw<T, KW>;
  constexpr int N4 = KW * R::RP / 4;
  constexpr int R4 = R::RP / 4;
  unsigned isum = 0;  // uint8: at most a few words per thread per batch
  for (int i = threadIdx.x; i < N4; i += Geo<KW>::NT) {
    const int r = i / R4, c4 = i - r * R4;
    if (4 * c4 >= R::FP) continue;
    const int o4 = (r * R::FP) / 4 + c4;
    const int gr = grow0 + r, gc = gcol0 + 4 * c4;
    const bool row_own = gr >= rlo && gr < rhi;
    float4 a, b;
    if constexpr (std::is_same<T, float>::value) {
      a = reinterpret_cast<const float4*>(rawx)[i];
      b = reinterpret_cast<const float4*>(rawy)[i];
      if (row_own) {
        const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (gc + j >= clo && gc + j < chi) {
            const float d = av[j] - bv[j];
            acc += (double)(d * d);
          }
      }
    } else if constexpr (std::is_same<T, unsigned char>::value) {
      const unsigned u = reinterpret_cast<const unsigned*>(rawx)[i];
      const unsigned v = reinterpret_cast<const unsigned*>(rawy)[i];
      if (row_own && gc + 3 >= clo && gc < chi) {
        unsigned d = __vabsdiffu4(u, v);
        if (gc < clo || gc + 3 >= chi) {  // a word across an ownership edge
          unsigned mask = 0;
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (gc + j >= clo && gc + j < chi) mask |= 0xffu << (8 * j);
          d &= mask;
        }
        isum = __dp4a(d, d, isum);
      }
      a = make_float4((float)(u & 0xff), (float)((u >> 8) & 0xff), (float)((u >> 16) & 0xff),
                      (float)(u >> 24));
      b = make_float4((float)(v & 0xff), (float)((v >> 8) & 0xff), (float)((v >> 16) & 0xff),
                      (float)(v >> 24));
    } else {
      const T* ex = rawx + 4 * i;
      const T* ey = rawy + 4 * i;
      a = make_float4(Ld<T>::f(ex[0]), Ld<T>::f(ex[1]), Ld<T>::f(ex[2]), Ld<T>::f(ex[3]));
      b = make_float4(Ld<T>::f(ey[0]), Ld<T>::f(ey[1]), Ld<T>::f(ey[2]), Ld<T>::f(ey[3]));
      if (row_own) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (gc + j >= clo && gc + j < chi) {
            if constexpr (std::is_same<T, double>::value) {
              const double d = ex[j] - ey[j];
              acc += d * d;
            } else if constexpr (std::is_same<T, unsigned short>::value) {
              const long long d = (long long)ex[j] - (long long)ey[j];
              acc += (unsigned long long)(d * d);
            } else {
              const float d = Ld<T>::f(ex[j]) - Ld<T>::f(ey[j]);
              acc += (double)(d * d);
            }
          }
      }
    }
    a.x -= p.shift; a.y -= p.shift; a.z -= p.shift; a.w -= p.shift;
    b.x -= p.shift; b.y -= p.shift; b.z -= p.shift; b.w -= p.shift;
    if constexpr (UV) {  // as stage_convert<T, KW, true>
      const float4 u = make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
      b = make_float4(a.x - b.x, a.y - b.y, a.z - b.z, a.w - b.w);
      a = u;
    }
    reinterpret_cast<float4*>(sx)[o4] = a;
    reinterpret_cast<float4*>(sy)[o4] = b;
  }
  if constexpr (std::is_same<T, unsigned char>::value) acc += isum;
}

// Register-path staging written straight to shared memory, element by
// element (no staging arrays stay live): LUMA projects RGB first; SQ also
// sums the owned squared differences of the unshifted values.
template <typename T, bool LUMA, bool SQ, int KW>
__device__ __forceinline__ void stage_direct(const SsimArgs& p, long long base, int row0,
                                             int col0, float* sx, float* sy, int rlo, int rhi,
                                             int clo, int chi, SqAcc<T>& acc) {
  using G = Geo<KW>;
  constexpr int FP = Raw<T, KW>::FP;
  const T* X = reinterpret_cast<const T*>(p.x);
  const T* Y = reinterpret_cast<const T*>(p.y);
#pragma unroll 4
  for (int e = 0; e < G::NE; ++e) {
    const int idx = threadIdx.x + e * G::NT;
    if (idx >= KW * G::SW) break;
    const int r = idx / G::SW;
    const int c = idx - r * G::SW;
    const int gr = row0 + r, gc = col0 + c;
    float a = 0.f, b = 0.f;
    if (gr >= 0 && gr < p.H && gc >= 0 && gc < p.W) {
      const long long o = base + (long long)gr * p.sh + gc;
      if constexpr (LUMA) {
        a = fmaf(p.lk0, Ld<T>::f(ldro(X + o)),
                 fmaf(p.lk1, Ld<T>::f(ldro(X + o + p.sc)),
                      fmaf(p.lk2, Ld<T>::f(ldro(X + o + 2 * p.sc)), p.lk3)));
        b = fmaf(p.lk0, Ld<T>::f(ldro(Y + o)),
                 fmaf(p.lk1, Ld<T>::f(ldro(Y + o + p.sc)),
                      fmaf(p.lk2, Ld<T>::f(ldro(Y + o + 2 * p.sc)), p.lk3)));
      } else {
        const T ra = ldro(X + o), rb = ldro(Y + o);
        a = Ld<T>::f(ra);
        b = Ld<T>::f(rb);
        if constexpr (SQ) {
          if (gr >= rlo && gr < rhi && gc >= clo && gc < chi) {
            if constexpr (std::is_same<T, unsigned char>::value ||
                          std::is_same<T, unsigned short>::value) {
              const long long d = (long long)ra - (long long)rb;
              acc += (unsigned long long)(d * d);
            } else if constexpr (std::is_same<T, double>::value) {
              const double d = ra - rb;
              acc += d * d;
            } else {
              const float d = a - b;
              acc += (double)(d * d);
            }
          }
        }
      }
      a -= p.shift;
      b -= p.shift;
    }
    sx[r * FP + c] = a;
    sy[r * FP + c] = b;
  }
}

// Last block, after the SSIM finaliser: per-plane squared-difference sums in a
// fixed order, then per-image and batch MSE and PSNR (bias - 10 log10 mse).
template <typename A>
static __device__ __noinline__ void sq_finalize(const SsimArgs& p, int bpp) {
  __shared__ A s_red[32];
  A* part = static_cast<A*>(p.part_sq);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int nw = blockDim.x >> 5;
  for (int pl = wid; pl < p.P; pl += nw) {
    A s = 0;
    for (int i = lane; i < bpp; i += 32) s += part[(long long)pl * bpp + i];
    s = warp_sum(s);
    if (lane == 0) part[(long long)pl * bpp] = s;
  }
  __syncthreads();
  __threadfence_block();
  const double per_img = (double)p.C * p.H * p.W;
  A t = 0;
  for (int n = threadIdx.x; n < p.N; n += blockDim.x) {
    A s = 0;
    for (int c = 0; c < p.C; ++c) s += part[(long long)(n * p.C + c) * bpp];
    const double mse = (double)s / per_img;
    if (p.out_mse_per_image) p.out_mse_per_image[n] = mse;
    if (p.out_psnr_per_image) p.out_psnr_per_image[n] = p.psnr_bias - 10.0 * log10(mse);
    if constexpr (std::is_same<A, unsigned long long>::value)
      if (p.out_ssd_per_image) p.out_ssd_per_image[n] = s;
    t += s;
  }
  t = block_sum(t, s_red);
  if (threadIdx.x == 0) {
    const double mse = (double)t / (per_img * p.N);
    if (p.out_mse_total) *p.out_mse_total = mse;
    if (p.out_psnr_total) *p.out_psnr_total = p.psnr_bias - 10.0 * log10(mse);
  }
}

// Last block: per-image GMS mean and GMSD (population std of q over the map
// positions of all the image's planes) from the per-block (sum d, sum d^2).
static __device__ __noinline__ void gm_fused_finalize(const SsimArgs& p, int bpp) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int nw = blockDim.x >> 5;
  const double npix = (double)p.gHo * p.gWo * p.Cm;
  for (int n = wid; n < p.N; n += nw) {
    double s = 0.0, s2 = 0.0;
    for (int c = 0; c < p.Cm; ++c) {
      const double* row = p.part_g + 2 * (long long)(n * p.Cm + c) * bpp;
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
      if (p.out_gms_per_image) p.out_gms_per_image[n] = 1.0 + md;
      if (p.out_gmsd_per_image) p.out_gmsd_per_image[n] = sqrt(var > 0.0 ? var : 0.0);
    }
  }
}

// Fused GMSD state of one thread.  Thread pair (2c, 2c+1) owns GMS map column
// j0 + c of its block, the even thread for x, the odd one for y, so all the
// block's warps share the work evenly.  Staged rows are visited in order; an
// even row's horizontal pair sums wait in e, an odd row completes a pooled
// row P, whose column difference D = P0 - P2 and 3-sum R = P0 + P1 + P2 enter
// a 3-row window kept as running sums: gx = D0 + D1 + D2 = d12 + D with
// d12 = D1 + D2 of the previous window, gy = R0 - R2.  Both are 3 x 4 times
// the pooled Prewitt responses (hence the 1/144); the pair exchanges them
// with one shuffle each and the even thread forms the map value.
struct GmState {
  float e0, e1, e2;
  float d2, d12;  // newest D, and D1 + D2
  float r1, r2;   // the two newest R
  float fs, fs2;
};

// One staged row (global input row r, this thread's six inputs at s[0..5]).
// Control flow is uniform across the block, so every lane reaches the
// shuffles.
__device__ __forceinline__ void gm_row(const SsimArgs& p, const float* s, int r, int rlo, int rhi,
                                       bool col_ok, GmState& g) {
  constexpr float K144 = 1.0f / 144.0f;
  if (r < rlo || r > rhi) return;
  const float h0 = s[0] + s[1], h1 = s[2] + s[3], h2 = s[4] + s[5];
  if ((r & 1) == 0) {
    g.e0 = h0; g.e1 = h1; g.e2 = h2;
    return;
  }
  const float P0 = g.e0 + h0, P1 = g.e1 + h1, P2 = g.e2 + h2;
  const float D = P0 - P2, R = P0 + P1 + P2;
  const float gx = g.d12 + D, gy = g.r1 - R;
  g.d12 = g.d2 + D;
  g.d2 = D;
  g.r1 = g.r2;
  g.r2 = R;
  if (r - rlo < 5) return;  // fewer than three pooled rows so far
  const float ox = __shfl_xor_sync(0xffffffffu, gx, 1);
  const float oy = __shfl_xor_sync(0xffffffffu, gy, 1);
  if (col_ok && (threadIdx.x & 1) == 0) {
    // the map value exactly as the GMSD kernel forms it (gmsd.cu)
    const float G1 = fmaf(fmaf(gx, gx, gy * gy), K144, p.geps);
    const float G2 = fmaf(fmaf(ox, ox, oy * oy), K144, p.geps);
    const float dG = fmaf(gx - ox, gx + ox, (gy - oy) * (gy + oy)) * K144;
    const float S = G1 + G2;
    const float G12 = G1 * G2;
    const float d = -__fdividef(dG * dG, (S + 2.f * G12 * rsqrtf(G12)) * (S + p.gT));
    g.fs += d;
    g.fs2 = fmaf(d, d, g.fs2);
  }
}

// The rows of one staged batch.  When every row lies inside the block's
// GMSD range with three pooled rows already in the window (the common case),
// each row is passed as the stand-in index 6 + its parity: in range, past the
// first five rows, and compile-time once the loop unrolls, so the batch
// becomes straight-line code.
template <int KW, int FP>
__device__ __forceinline__ void gm_batch(const SsimArgs& p, const float* s, int row0, int rlo,
                                         int rhi, bool col_ok, GmState& g) {
  if (row0 - rlo >= 5 && row0 + KW - 1 <= rhi) {
    if (row0 & 1) {
#pragma unroll
      for (int k = 0; k < KW; ++k) gm_row(p, s + k * FP, 6 + ((k + 1) & 1), 0, 1 << 30, col_ok, g);
    } else {
#pragma unroll
      for (int k = 0; k < KW; ++k) gm_row(p, s + k * FP, 6 + (k & 1), 0, 1 << 30, col_ok, g);
    }
    return;
  }
#pragma unroll 1
  for (int k = 0; k < KW; ++k) gm_row(p, s + k * FP, row0 + k, rlo, rhi, col_ok, g);
}

template <typename T, int KW, bool CS, int STAGE, bool SQ, bool GM = false>
__device__ __forceinline__ void ssim_fwd_body(const SsimArgs& p) {
  using G = Geo<KW>;
  using R = Raw<T, KW>;
  constexpr bool TMA = (STAGE == STAGE_TMA);
  // TMA staging (except under the fused GMSD state, which reads x' and y')
  // stages the rows as u = x' + y', v = x' - y'
  constexpr bool UV = TMA && !GM;
  extern __shared__ __align__(128) float4 smem4[];
  float4* sH = smem4;                                        // [KW][NT]
  float* sX = reinterpret_cast<float*>(smem4 + KW * G::NT);  // [KW][FP]
  float* sY = sX + KW * R::FP;
  T* rawX = R::kInPlace ? reinterpret_cast<T*>(sX)
                        : reinterpret_cast<T*>(reinterpret_cast<char*>(sX) + R::kFloatBytes);
  T* rawY = R::kInPlace ? reinterpret_cast<T*>(sY) : rawX + KW * R::RP;
  __shared__ double s_red[32];
  __shared__ int s_flag;
  __shared__ __align__(8) unsigned long long s_bar;

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
  float* map = p.map_out ? p.map_out + (long long)plane * p.Hout * p.Wout : nullptr;
  // TMA x coordinate of the strip, rounded down to 16 bytes, and the offset of
  // column c0 inside the staged rows
  const int xm = c0 + p.tma_d;
  const int x0 = TMA ? (xm / R::XA) * R::XA : 0;
  const int sofs = TMA ? xm - x0 : 0;

  if constexpr (TMA) {
    if (t == 0) mbar_init(&s_bar, 1);
    fence_async_smem();
    __syncthreads();
    stage_tma<T, KW>(p, pn, pc, r0, x0, rawX, rawY, &s_bar);
  }

  float4 ring[KW];
#pragma unroll
  for (int k = 0; k < KW; ++k) ring[k] = make_float4(0.f, 0.f, 0.f, 0.f);
  double acc_s = 0.0, acc_cs = 0.0;
  // SQ: input pixels this block owns for the squared-difference sums (the
  // last strip / chunk also owns the K-1 columns / rows past the map)
  SqAcc<T> acc_sq = 0;
  const int sq_chi = (blockIdx.x == gridDim.x - 1) ? p.W : c0 + G::NT;
  const int sq_rhi = (blockIdx.y == gridDim.y - 1) ? p.H : r0 + rows;
  // GM: this block's GMS map rows are those i with 2i in [r0, r0 + rows) (the
  // last chunk: all from there on), which need input rows [2 i_lo, 2 i_hi + 5]
  GmState gst{};
  int g_rlo = 0, g_rhi = -1;
  bool g_col = false;
  if constexpr (GM) {
    const int i_lo = (r0 + 1) >> 1;
    const int i_end = (blockIdx.y == gridDim.y - 1) ? p.gHo : (r0 + rows + 1) >> 1;
    g_rlo = 2 * i_lo;
    g_rhi = i_end > i_lo ? 2 * (i_end - 1) + 5 : -1;
    g_col = (c0 >> 1) + (t >> 1) < p.gWo;
  }
  const float* gm_in = ((t & 1) ? sY : sX) + sofs + 2 * (t >> 1);

  for (int m = 0; m < iters; ++m) {
    if constexpr (!TMA) {
      // direct staging: nothing stays live across the compute (the block's
      // second resident copy hides the load latency); the previous batch's
      // horizontal pass ended at a barrier
      stage_direct<T, STAGE == STAGE_LUMA, SQ, KW>(p, base, r0 + m * KW, c0, sX, sY, r0, sq_rhi,
                                                   c0, sq_chi, acc_sq);
    }
    if constexpr (TMA) {
      mbar_wait(&s_bar, m & 1, p.err);
      if constexpr (SQ)
        stage_convert_sq<T, KW, UV>(p, rawX, rawY, sX, sY, r0 + m * KW, x0 - p.tma_d, r0, sq_rhi,
                                    c0, sq_chi, acc_sq);
      else
        stage_convert<T, KW, UV>(p, rawX, rawY, sX, sY);
    }
    __syncthreads();
    // horizontal: warp k -> staged row k, lane -> columns [lane*KW, lane*KW+KW)
    {
      const float* rx = sX + warp * R::FP + sofs + lane * KW;
      const float* ry = sY + warp * R::FP + sofs + lane * KW;
      float4* out = sH + warp * G::NT + lane * KW;
      hblur4<KW, TMA, UV>(p, rx, ry, out);  // TMA staging implies symmetric taps
    }
    // GM: the staged rows through the GMSD state; the next batch's copy and
    // convert rewrite sX / sY only after the barrier below
    if constexpr (GM) gm_batch<KW, R::FP>(p, gm_in, r0 + m * KW, g_rlo, g_rhi, g_col, gst);
    __syncthreads();
    const bool more = (m + 1 < iters);
    if constexpr (TMA) {
      if (more) stage_tma<T, KW>(p, pn, pc, r0 + (m + 1) * KW, x0, rawX, rawY, &s_bar);
    }
    // vertical + epilogue; interior batches (every slot a map row of this
    // chunk) skip the per-row tests
    float fs = 0.f, fcs = 0.f;
    // FLAT: an interior batch with no map to write.  Every slot is a map row
    // of this chunk, so the rows are computed without branches and a column
    // past the map adds zero (a select, not a branch).
    auto rows_step = [&](auto chk, auto flat) {
      constexpr bool CHK = decltype(chk)::value;
      constexpr bool FLAT = decltype(flat)::value;
#pragma unroll
      for (int k = 0; k < KW; ++k) {
        ring[k] = sH[k * G::NT + t];
        const int o = m * KW + k - (KW - 1);
        if (FLAT || (col_ok && (!CHK || (o >= 0 && o < rows)))) {
          float S, cs = 0.f;
          if constexpr (UV) {
            const SsimCs v = ssim_uv<CS>(p, vblur_at<KW, 4, TMA>(p, ring, k));
            S = v.S;
            cs = v.cs;
          } else {
            const Moments mo = moments(p, vblur_at<KW, 4, TMA>(p, ring, k));
            // one approximate reciprocal (a few ulp) for S = A1 A2 / (B1 B2) and
            // cs = A2 / B2 = A2 B1 / (B1 B2)
            const float inv = __fdividef(1.0f, mo.B1 * mo.B2);
            S = mo.A1 * mo.A2 * inv;
            if (CS) cs = mo.A2 * mo.B1 * inv;
          }
          if (FLAT) {
            fs += col_ok ? S : 0.f;
            if (CS) fcs += col_ok ? cs : 0.f;
          } else {
            fs += S;
            if (CS) fcs += cs;
            if (map) map[(long long)(r0 + o) * p.Wout + col] = S;
          }
        }
      }
    };
    const int o_first = m * KW - (KW - 1);
    if (o_first >= 0 && o_first + KW - 1 < rows) {
      if (map) rows_step(std::false_type{}, std::false_type{});
      else rows_step(std::false_type{}, std::true_type{});
    } else {
      rows_step(std::true_type{}, std::false_type{});
    }
    acc_s += (double)fs;
    acc_cs += (double)fcs;
  }

  const int bpp = p.strips * p.chunks;
  const long long pidx = (long long)plane * bpp + blockIdx.y * p.strips + blockIdx.x;
  acc_s = block_sum(acc_s, s_red);
  if (t == 0) p.part_s[pidx] = acc_s;
  if (CS) {
    acc_cs = block_sum(acc_cs, s_red);
    if (t == 0) p.part_cs[pidx] = acc_cs;
  }
  if constexpr (SQ) {
    __shared__ SqAcc<T> s_red_q[32];
    acc_sq = block_sum(acc_sq, s_red_q);
    if (t == 0) static_cast<SqAcc<T>*>(p.part_sq)[pidx] = acc_sq;
  }
  if constexpr (GM) {
    // a thread's column sums stay in float (a few hundred small terms, kept
    // there to stay within 80 registers); the block sums are double
    double acc_g = block_sum((double)gst.fs, s_red);
    double acc_g2 = block_sum((double)gst.fs2, s_red);
    // part_g is only 8-byte aligned (it follows 3 x nb doubles): two stores
    if (t == 0) {
      p.part_g[2 * pidx] = acc_g;
      p.part_g[2 * pidx + 1] = acc_g2;
    }
  }
  if (last_block_arrived(p.counter, gridDim.x * gridDim.y * gridDim.z, &s_flag)) {
    if constexpr (GM) {
      gm_fused_finalize(p, bpp);
      __syncthreads();
    }
    ssim_fwd_finalize(p, bpp);
    if constexpr (SQ) {
      __syncthreads();
      sq_finalize<SqAcc<T>>(p, bpp);
    }
  }
}

// DW: taps from `wdev` (register staging only; see load_device_taps).
template <typename T, int KW, bool CS, int STAGE, bool SQ = false, bool DW = false>
__global__ void __launch_bounds__(32 * KW, 2) ssim_fwd_kernel(const __grid_constant__ SsimArgs p) {
  if constexpr (DW) {
    static_assert(STAGE == STAGE_GENERIC, "device taps use register staging");
    SsimArgs q = p;
    load_device_taps<KW>(q);
    ssim_fwd_body<T, KW, CS, STAGE, SQ>(q);
  } else {
    ssim_fwd_body<T, KW, CS, STAGE, SQ>(p);
  }
}

// SSIM with GMSD of the same pair from the same staged rows
// (ssim_gmsd_fusable).  Two blocks per SM as the plain kernel; the GMSD state
// needs 88 registers a thread instead of 80 (88 x 352 x 2 fits an SM).
template <typename T, int KW, bool SQ>
__global__ void __launch_bounds__(32 * KW, 2) ssim_gmsd_kernel(const __grid_constant__ SsimArgs p) {
  ssim_fwd_body<T, KW, false, STAGE_TMA, SQ, true>(p);
}

template <typename T, int KW, int STAGE>
static constexpr size_t fwd_smem() {
  return sizeof(float4) * KW * Geo<KW>::NT + Raw<T, KW>::kFloatBytes +
         (STAGE == STAGE_TMA ? Raw<T, KW>::kRawBytes : 0);
}

template <typename T, int KW, bool CS, int STAGE, bool SQ = false, bool DW = false,
          bool GM = false>
static int launch_fwd(const SsimArgs& p, int device, cudaStream_t st) {
  static_assert(!GM || (STAGE == STAGE_TMA && !CS && !DW), "GMSD rides on the TMA forward");
  auto kern = [] {
    if constexpr (GM) return ssim_gmsd_kernel<T, KW, SQ>;
    else return ssim_fwd_kernel<T, KW, CS, STAGE, SQ, DW>;
  }();
  const size_t sm = fwd_smem<T, KW, STAGE>();
  static bool done[64] = {false};
  FAB_TRY(ensure_smem(kern, sm, device, done));
  dim3 grid(p.strips, p.chunks, p.P);
  kern<<<grid, 32 * KW, sm, st>>>(p);
  FAB_LAUNCH_CHECK();
  return FA_OK;
}

}  // namespace fab
