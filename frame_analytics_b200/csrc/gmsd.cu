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
#include "ssim_common.cuh"  // TMA/mbarrier helpers and make_row_map

namespace fab {

constexpr int GM_T = 256;             // threads
constexpr int GM_CPT = 2;             // pooled columns per thread
constexpr int GM_DW = GM_T * GM_CPT;  // pooled columns staged per strip
constexpr int GM_OW = GM_DW - 4;      // output columns per strip (a multiple of 4 keeps
                                      // every strip's 8-byte uint8 loads aligned)
constexpr int GM_R = 6;               // output rows per iteration
constexpr int GM_RING = GM_R + 2;

struct GmsdArgs {
  CUtensorMap tmx, tmy;  // TMA row maps (uint8 TMA kernel)
  int tma_d;             // leading elements the aligned map base adds
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
  unsigned int* err;  // host-mapped error word of the bounded waits
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
    if (dc + GM_CPT <= p.Wd && ((reinterpret_cast<uintptr_t>(b0) | reinterpret_cast<uintptr_t>(b1)) & 3u) == 0) {
      const unsigned u0 = __ldg(reinterpret_cast<const unsigned*>(b0));
      const unsigned u1 = __ldg(reinterpret_cast<const unsigned*>(b1));
#pragma unroll
      for (int i = 0; i < GM_CPT; ++i) {
        const unsigned wa = u0 >> (i * 16), wb = u1 >> (i * 16);
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

// One staged pooled row at this thread's columns c .. c+3: column differences
// D[j] = s[j] - s[j+2] and 3-sums R[j] = s[j] + s[j+1] + s[j+2].
__device__ __forceinline__ void gm_row_terms(const float* s, float (&D)[GM_CPT],
                                             float (&R)[GM_CPT]) {
  static_assert(GM_CPT == 2, "4 staged floats cover 2 output columns");
  const float2 a = *reinterpret_cast<const float2*>(s);  // 8-byte aligned: s = row + 2t
  const float2 b = *reinterpret_cast<const float2*>(s + 2);
  const float v[4] = {a.x, a.y, b.x, b.y};
#pragma unroll
  for (int j = 0; j < GM_CPT; ++j) {
    D[j] = v[j] - v[j + 2];
    R[j] = v[j] + v[j + 1] + v[j + 2];
  }
}

// Output rows 0..nr-1 of one iteration from pooled rows 0..nr+1 of a ring
// (row pitch `pitch` floats): this thread's GM_CPT columns, summed into
// fs (d = q - 1) and fs2 (d^2); the map is written when requested.
template <bool MAP>
__device__ __forceinline__ void gm_rows(const GmsdArgs& p, const float* sxr, const float* syr,
                                        int pitch, int nr, int t, int dc0, int plane, int orow0,
                                        float& fs, float& fs2) {
    const int c0t = t * GM_CPT;
    constexpr float NINTH = 1.0f / 9.0f;
    // output columns of this thread inside the strip and the map
    const int ncol = min(min(GM_OW, p.Wout - dc0) - c0t, GM_CPT);
    // Sliding 3-row window of column differences D (for gx) and row sums R
    // (for gy) of this thread's 4 output columns, per image; the ring slot
    // of pooled row r is r % 3, static because the loop is unrolled.
    float Dx[3][GM_CPT], Rx[3][GM_CPT], Dy[3][GM_CPT], Ry[3][GM_CPT];
#pragma unroll
    for (int r = 0; r < GM_R + 2; ++r) {
      if (r < nr + 2) {
        gm_row_terms(sxr + r * pitch + c0t, Dx[r % 3], Rx[r % 3]);
        gm_row_terms(syr + r * pitch + c0t, Dy[r % 3], Ry[r % 3]);
        if (r >= 2) {
          const int k = r - 2, s0 = (r - 2) % 3, s1 = (r - 1) % 3, s2 = r % 3;
#pragma unroll
          for (int i = 0; i < GM_CPT; ++i) {
            const int c = c0t + i;
            if (i < ncol) {
              // 3x the Prewitt/3 responses
              const float gx1 = Dx[s0][i] + Dx[s1][i] + Dx[s2][i], gy1 = Rx[s0][i] - Rx[s2][i];
              const float gx2 = Dy[s0][i] + Dy[s1][i] + Dy[s2][i], gy2 = Ry[s0][i] - Ry[s2][i];
              const float G1 = fmaf(fmaf(gx1, gx1, gy1 * gy1), NINTH, p.eps);  // g1^2
              const float G2 = fmaf(fmaf(gx2, gx2, gy2 * gy2), NINTH, p.eps);  // g2^2
              // G1 - G2 from differences and sums of the gradients: no cancellation
              const float dG = fmaf(gx1 - gx2, gx1 + gx2, (gy1 - gy2) * (gy1 + gy2)) * NINTH;
              const float S = G1 + G2;
              // q - 1 = -(g1 - g2)^2 / (g1^2 + g2^2 + T),  (g1 - g2)^2 = dG^2 / (g1 + g2)^2.
              // g1 g2 = G12 rsqrt(G12) (G12 >= eps^2 > 0) and one approximate
              // division: a few ulp of d, which is small where q is near 1
              const float G12 = G1 * G2;
              const float d = -__fdividef(dG * dG, (S + 2.f * G12 * rsqrtf(G12)) * (S + p.T));
              fs += d;
              fs2 = fmaf(d, d, fs2);
              if constexpr (MAP)
                p.map[((long long)plane * p.Hout + (orow0 + k)) * p.Wout + dc0 + c] = 1.0f + d;
            }
          }
        }
      }
    }
}

// gm_rows for the uint8 TMA kernel: the ring holds (x, y) pairs per column
// (float2), as exact integer 2x2 sums (DOWN) or bytes, so both images go
// through the Prewitt sums and g^2 in packed f32x2 instructions.  The 1/4 of
// the pool and the 1/3 of Prewitt are folded into K = 1/144 (1/9 without the
// pool); integer inputs keep gx, gy exact.
template <bool MAP, bool DOWN>
__device__ __forceinline__ void gm_rows_packed(const GmsdArgs& p, const float2* ring, int pitch,
                                               int nr, int t, int dc0, int plane, int orow0,
                                               float& fs, float& fs2) {
  static_assert(GM_CPT == 2, "two output columns per thread");
  constexpr float K = DOWN ? 1.0f / 144.0f : 1.0f / 9.0f;
  const int c0t = t * GM_CPT;
  const int ncol = min(min(GM_OW, p.Wout - dc0) - c0t, GM_CPT);
  const float2 kk = make_float2(K, K), ee = make_float2(p.eps, p.eps);
  const float2 m1 = make_float2(-1.f, -1.f);
  float2 D[3][GM_CPT], R[3][GM_CPT];  // column differences / 3-sums, ring slot r % 3
#pragma unroll
  for (int r = 0; r < GM_R + 2; ++r) {
    if (r < nr + 2) {
      const float2* rowp = ring + r * pitch;
      const float4 A = *reinterpret_cast<const float4*>(rowp + c0t);
      const float4 B = *reinterpret_cast<const float4*>(rowp + c0t + 2);
      const float2 P0 = make_float2(A.x, A.y), P1 = make_float2(A.z, A.w);
      const float2 P2 = make_float2(B.x, B.y), P3 = make_float2(B.z, B.w);
      D[r % 3][0] = __ffma2_rn(P2, m1, P0);
      D[r % 3][1] = __ffma2_rn(P3, m1, P1);
      const float2 s12 = __fadd2_rn(P1, P2);
      R[r % 3][0] = __fadd2_rn(P0, s12);
      R[r % 3][1] = __fadd2_rn(s12, P3);
      if (r >= 2) {
        const int k = r - 2, s0 = (r - 2) % 3, s1 = (r - 1) % 3, s2 = r % 3;
#pragma unroll
        for (int i = 0; i < GM_CPT; ++i) {
          if (i < ncol) {
            const float2 gx = __fadd2_rn(__fadd2_rn(D[s0][i], D[s1][i]), D[s2][i]);
            const float2 gy = __ffma2_rn(R[s2][i], m1, R[s0][i]);
            const float2 G = __ffma2_rn(__ffma2_rn(gx, gx, __fmul2_rn(gy, gy)), kk, ee);
            // G1 - G2 from differences and sums of the gradients: no cancellation
            const float dG = fmaf(gx.x - gx.y, gx.x + gx.y, (gy.x - gy.y) * (gy.x + gy.y)) * K;
            const float S = G.x + G.y;
            const float G12 = G.x * G.y;
            const float d = -__fdividef(dG * dG, (S + 2.f * G12 * rsqrtf(G12)) * (S + p.T));
            fs += d;
            fs2 = fmaf(d, d, fs2);
            if constexpr (MAP)
              p.map[((long long)plane * p.Hout + (orow0 + k)) * p.Wout + dc0 + c0t + i] = 1.0f + d;
          }
        }
      }
    }
  }
}

// Prewitt window of the uint8 TMA kernel carried across iterations: per
// output column, (x, y) pairs of the newest column difference D, of D1 + D2
// (the two newest), and of the two newest 3-sums R.  gx = D0 + D1 + D2 and
// gy = R0 - R2 then need one add each, and no pooled row is pooled or read
// twice (the ring holds only new rows after the first iteration).
struct GmWin {
  float2 d2[GM_CPT], d12[GM_CPT], r1[GM_CPT], r2[GM_CPT];
};

// Ring rows 0..n-1 hold pooled rows g0 .. g0+n-1 of the block (g counted from
// the block's first pooled row); a map row is emitted from pooled row g >= 2
// (map row r0 + g - 2).
template <bool MAP, bool DOWN, int NR = GM_R + 2>
__device__ __forceinline__ void gm_rows_window(const GmsdArgs& p, const float2* ring, int pitch,
                                               int n, int g0, int t, int dc0, int plane, int r0,
                                               GmWin& w, float& fs, float& fs2) {
  static_assert(GM_CPT == 2, "two output columns per thread");
  constexpr float K = DOWN ? 1.0f / 144.0f : 1.0f / 9.0f;
  const int c0t = t * GM_CPT;
  const int ncol = min(min(GM_OW, p.Wout - dc0) - c0t, GM_CPT);
  const float2 kk = make_float2(K, K), ee = make_float2(p.eps, p.eps);
  const float2 m1 = make_float2(-1.f, -1.f);
#pragma unroll
  for (int q = 0; q < NR; ++q) {
    if (q < n) {
      const float2* rowp = ring + q * pitch;
      const float4 A = *reinterpret_cast<const float4*>(rowp + c0t);
      const float4 B = *reinterpret_cast<const float4*>(rowp + c0t + 2);
      const float2 P0 = make_float2(A.x, A.y), P1 = make_float2(A.z, A.w);
      const float2 P2 = make_float2(B.x, B.y), P3 = make_float2(B.z, B.w);
      const float2 s12 = __fadd2_rn(P1, P2);
      const float2 D[GM_CPT] = {__ffma2_rn(P2, m1, P0), __ffma2_rn(P3, m1, P1)};
      const float2 R[GM_CPT] = {__fadd2_rn(P0, s12), __fadd2_rn(s12, P3)};
      const bool emit = g0 + q >= 2;
#pragma unroll
      for (int i = 0; i < GM_CPT; ++i) {
        const float2 gx = __fadd2_rn(w.d12[i], D[i]);
        const float2 gy = __ffma2_rn(R[i], m1, w.r1[i]);
        w.d12[i] = __fadd2_rn(w.d2[i], D[i]);
        w.d2[i] = D[i];
        w.r1[i] = w.r2[i];
        w.r2[i] = R[i];
        if (emit && i < ncol) {
          const float2 G = __ffma2_rn(__ffma2_rn(gx, gx, __fmul2_rn(gy, gy)), kk, ee);
          // G1 - G2 from differences and sums of the gradients: no cancellation
          const float dG = fmaf(gx.x - gx.y, gx.x + gx.y, (gy.x - gy.y) * (gy.x + gy.y)) * K;
          const float S = G.x + G.y;
          const float G12 = G.x * G.y;
          const float d = -__fdividef(dG * dG, (S + 2.f * G12 * rsqrtf(G12)) * (S + p.T));
          fs += d;
          fs2 = fmaf(d, d, fs2);
          if constexpr (MAP)
            p.map[((long long)plane * p.Hout + (r0 + g0 + q - 2)) * p.Wout + dc0 + c0t + i] =
                1.0f + d;
        }
      }
    }
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

template <typename T, bool DOWN, bool LUMA, bool MAP>
__global__ void __launch_bounds__(GM_T, 2) gmsd_kernel(GmsdArgs p) {
  __shared__ __align__(16) float sx[GM_RING][GM_DW + 4];
  __shared__ __align__(16) float sy[GM_RING][GM_DW + 4];
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
    // pooled rows rb+2 .. rb+nr+1 into ring rows 2 .. nr+1: every row's loads
    // are issued before the first store, so the iteration pays one memory
    // latency, not GM_R of them
    {
      float a[GM_R][GM_CPT], b[GM_R][GM_CPT];
#pragma unroll
      for (int k = 0; k < GM_R; ++k) {
        if (k < nr) {
          const int dr = r0 + rb + 2 + k;
          gm_load4<T, DOWN, LUMA>(p, X, base, dr, dc, a[k]);
          gm_load4<T, DOWN, LUMA>(p, Y, base, dr, dc, b[k]);
        }
      }
#pragma unroll
      for (int k = 0; k < GM_R; ++k) {
        if (k < nr) {
#pragma unroll
          for (int i = 0; i < GM_CPT; ++i) {
            sx[2 + k][t * GM_CPT + i] = a[k][i];
            sy[2 + k][t * GM_CPT + i] = b[k][i];
          }
        }
      }
    }
    __syncthreads();
    float fs = 0.f, fs2 = 0.f;
    gm_rows<MAP>(p, &sx[0][0], &sy[0][0], GM_DW + 4, nr, t, dc0, plane, r0 + rb, fs, fs2);
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
// uint8 kernel with TMA staging.  The first iteration stages GM_R + 2 pooled
// rows (2 * (GM_R + 2) input rows with the 2x2 pool), every later one the next
// GM_R: the Prewitt window is carried in registers (GmWin), so no input row
// is copied, pooled or differenced twice.  Rows arrive as one-row TMA boxes
// (GMT_BOX bytes, x rounded down to 16 bytes), issued by all threads; the
// block pools them from shared memory into the float ring, issues the next
// iteration's copies, then computes.  No thread waits on a global load.
// ---------------------------------------------------------------------------
constexpr int GMT_BOX = 256;

template <bool DOWN>
struct GmTma {
  static constexpr int RIN = DOWN ? 2 * (GM_R + 2) : (GM_R + 2);  // input rows / iteration
  static constexpr int NB = DOWN ? 5 : 3;                         // boxes per input row
  static constexpr int IW = NB * GMT_BOX;                         // staged bytes per row
  static constexpr unsigned TX = 2u * RIN * IW;                   // bytes per iteration
  static constexpr int RP = GM_DW + 4;                            // ring pitch, floats
  static constexpr size_t RAW = (size_t)2 * RIN * IW;
  static constexpr size_t SMEM = RAW + sizeof(float2) * (GM_R + 2) * RP;
  static_assert(RAW % 128 == 0, "ring must stay 16-byte aligned");
};

// 4 (or 8) consecutive bytes at byte offset o of a staged row, any alignment.
__device__ __forceinline__ unsigned gm_bytes4(const unsigned char* row, int o) {
  const unsigned* w = reinterpret_cast<const unsigned*>(row) + (o >> 2);
  return __funnelshift_r(w[0], w[1], (o & 3) * 8);
}

// Rows q < n (n <= NR) of the staged bytes pooled (or converted) into the
// (x, y) float ring of the uint8 TMA kernel: exact integer 2x2 sums by dp4a
// (the 1/4 is folded into the Prewitt constant).
template <bool DOWN, int NR>
__device__ __forceinline__ void gm_pool_rows(const unsigned char* rawx, const unsigned char* rawy,
                                             float2* ring, int sofs, int t, int n) {
  using G = GmTma<DOWN>;
  const bool al4 = (sofs & 3) == 0;  // uniform: staged words are aligned
#pragma unroll
  for (int q = 0; q < NR; ++q) {
    if (q < n) {
      float4 v;
      if (DOWN) {
        const int o = sofs + 4 * t;
        const unsigned char* x0r = rawx + (2 * q) * G::IW;
        const unsigned char* y0r = rawy + (2 * q) * G::IW;
        unsigned ax, bx, ay, by;
        if (al4) {
          ax = *reinterpret_cast<const unsigned*>(x0r + o);
          bx = *reinterpret_cast<const unsigned*>(x0r + G::IW + o);
          ay = *reinterpret_cast<const unsigned*>(y0r + o);
          by = *reinterpret_cast<const unsigned*>(y0r + G::IW + o);
        } else {
          ax = gm_bytes4(x0r, o);
          bx = gm_bytes4(x0r + G::IW, o);
          ay = gm_bytes4(y0r, o);
          by = gm_bytes4(y0r + G::IW, o);
        }
        constexpr unsigned LO = 0x00000101u, HI = 0x01010000u;
        v = make_float4((float)__dp4a(ax, LO, __dp4a(bx, LO, 0u)),
                        (float)__dp4a(ay, LO, __dp4a(by, LO, 0u)),
                        (float)__dp4a(ax, HI, __dp4a(bx, HI, 0u)),
                        (float)__dp4a(ay, HI, __dp4a(by, HI, 0u)));
      } else {
        const unsigned a = gm_bytes4(rawx + q * G::IW, sofs + 2 * t);
        const unsigned b = gm_bytes4(rawy + q * G::IW, sofs + 2 * t);
        v = make_float4((float)(a & 0xff), (float)(b & 0xff), (float)((a >> 8) & 0xff),
                        (float)((b >> 8) & 0xff));
      }
      reinterpret_cast<float4*>(ring + q * G::RP)[t] = v;
    }
  }
}

template <bool DOWN, bool MAP>
__global__ void __launch_bounds__(GM_T, 3) gmsd_tma_kernel(const __grid_constant__ GmsdArgs p) {
  using G = GmTma<DOWN>;
  extern __shared__ __align__(128) unsigned char s_gm[];
  unsigned char* rawx = s_gm;
  unsigned char* rawy = s_gm + G::RIN * G::IW;
  float2* ring = reinterpret_cast<float2*>(s_gm + G::RAW);  // [GM_R+2][RP] (x, y) pairs
  __shared__ __align__(8) unsigned long long s_bar;
  __shared__ double s_red[32];
  __shared__ int s_flag;

  const int t = threadIdx.x;
  const int plane = blockIdx.z;
  const int pn = plane / p.Cm, pc = plane - pn * p.Cm;
  const int dc0 = blockIdx.x * GM_OW;
  const int r0 = blockIdx.y * p.RH;
  const int rows = min(p.RH, p.Hout - r0);
  const int xin = (DOWN ? 2 * dc0 : dc0) + p.tma_d;
  const int x0 = (xin / 16) * 16, sofs = xin - x0;

  // The block needs pooled rows [r0, r0 + rows + 2).  Iteration 0 stages
  // GM_R + 2 of them, every later one the next GM_R; the Prewitt window
  // carries the two rows before each iteration's first in registers.
  constexpr int PR = DOWN ? 2 : 1;  // input rows per pooled row
  const int np_total = rows + 2;
  auto first_of = [&](int it) { return it == 0 ? 0 : 2 + it * GM_R; };
  auto count_of = [&](int it) {
    const int f = first_of(it);
    return min(it == 0 ? GM_R + 2 : GM_R, np_total - f);
  };
  auto issue = [&](int it) {
    const int f = first_of(it), n = count_of(it);
    const int rin = PR * n;
    if (t == 0) mbar_expect_tx(&s_bar, 2u * rin * G::IW);
    fence_async_smem();
    for (int i = t; i < 2 * rin * G::NB; i += GM_T) {
      const int img = i / (rin * G::NB), rem = i - img * (rin * G::NB);
      const int row = rem / G::NB, box = rem - row * G::NB;
      const int in_row = PR * (r0 + f) + row;
      unsigned char* dst = (img ? rawy : rawx) + row * G::IW + box * GMT_BOX;
      tma_row(dst, img ? &p.tmy : &p.tmx, x0 + box * GMT_BOX, in_row, pc, pn, &s_bar);
    }
  };

  if (t == 0) mbar_init(&s_bar, 1);
  fence_async_smem();
  __syncthreads();
  issue(0);

  GmWin win{};
  double acc = 0.0, acc2 = 0.0;
  for (int it = 0; first_of(it) < np_total; ++it) {
    const int g0 = first_of(it), n = count_of(it);
    mbar_wait(&s_bar, it & 1, p.err);
    // pool (or convert) the staged bytes into the ring: exact integer 2x2
    // sums by dp4a (the 1/4 is folded into the Prewitt constant).  The row
    // count is a compile-time bound for the first (GM_R + 2) and the steady
    // (GM_R) iterations, so no predicated-off row is issued there.
    if (n == GM_R + 2) gm_pool_rows<DOWN, GM_R + 2>(rawx, rawy, ring, sofs, t, n);
    else if (n == GM_R) gm_pool_rows<DOWN, GM_R>(rawx, rawy, ring, sofs, t, n);
    else gm_pool_rows<DOWN, GM_R + 2>(rawx, rawy, ring, sofs, t, n);
    __syncthreads();
    if (first_of(it + 1) < np_total) issue(it + 1);  // the staging buffer is free again
    float fs = 0.f, fs2 = 0.f;
    if (n == GM_R + 2)
      gm_rows_window<MAP, DOWN, GM_R + 2>(p, ring, G::RP, n, g0, t, dc0, plane, r0, win, fs, fs2);
    else if (n == GM_R)
      gm_rows_window<MAP, DOWN, GM_R>(p, ring, G::RP, n, g0, t, dc0, plane, r0, win, fs, fs2);
    else
      gm_rows_window<MAP, DOWN, GM_R + 2>(p, ring, G::RP, n, g0, t, dc0, plane, r0, win, fs, fs2);
    acc += (double)fs;
    acc2 += (double)fs2;
    __syncthreads();  // the ring is rewritten next iteration
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
// uint8, 2x2 pool, no map: register streaming.  One warp owns a strip of 128
// pooled columns (256 input bytes per row: two 128-byte lines) and walks down
// a chunk of rows; lane l pools columns 4l .. 4l + 3 from one 8-byte load per
// input row and image, takes columns 4l + 4 and 4l + 5 from lane l + 1 by
// shuffle, and emits map columns 4l .. 4l + 3 (lanes 0..30: a strip emits
// 124 columns, so strips start 248 bytes apart and every load stays 8-byte
// aligned).  The Prewitt window is carried in registers (the GmWin
// recurrence), the loads of the next two pooled rows are in flight while the
// current two are computed, and nothing goes through shared memory until the
// block's final sums.  Pool sums come out of dp4a with 2^23's float bits as
// the addend, so one packed subtract makes them floats (no conversions).
// ---------------------------------------------------------------------------
constexpr int GR_T = 256;                 // threads: 8 warps, one strip each
constexpr int GR_WARPS = GR_T / 32;
constexpr int GR_OW = 124;                // map columns per strip
constexpr int GR_PER_SM = 2;              // resident blocks per SM (registers)

struct GrRows {
  uint2 x0, x1, y0, y1;  // one pooled row: two input rows of both images
};

// One pooled row: the Prewitt window update of this lane's four columns and,
// when EMIT, their map values (d = q - 1) added to fs / fs2 (columns at or
// past ncol masked; TK = T * 144^2).  Pool sums come out of dp4a with 2^23's float bits as
// the addend, so one packed subtract makes them floats.
template <bool EMIT>
__device__ __forceinline__ void gr_step(const GrRows& v, float2 (&d2)[4], float2 (&d12)[4],
                                        float2 (&r1)[4], float2 (&r2)[4], int ncol, float TK,
                                        float2 ee, float& fs, float& fs2) {
  constexpr unsigned LO = 0x00000101u, HI = 0x01010000u, M = 0x4B000000u;
  constexpr float K = 1.0f / 144.0f, KI2 = 144.0f * 144.0f;
  const float2 kk = make_float2(K, K), m1 = make_float2(-1.f, -1.f);
  const float2 nmag = make_float2(-8388608.f, -8388608.f);
  float2 P[6];
  P[0] = make_float2(__uint_as_float(__dp4a(v.x0.x, LO, __dp4a(v.x1.x, LO, M))),
                     __uint_as_float(__dp4a(v.y0.x, LO, __dp4a(v.y1.x, LO, M))));
  P[1] = make_float2(__uint_as_float(__dp4a(v.x0.x, HI, __dp4a(v.x1.x, HI, M))),
                     __uint_as_float(__dp4a(v.y0.x, HI, __dp4a(v.y1.x, HI, M))));
  P[2] = make_float2(__uint_as_float(__dp4a(v.x0.y, LO, __dp4a(v.x1.y, LO, M))),
                     __uint_as_float(__dp4a(v.y0.y, LO, __dp4a(v.y1.y, LO, M))));
  P[3] = make_float2(__uint_as_float(__dp4a(v.x0.y, HI, __dp4a(v.x1.y, HI, M))),
                     __uint_as_float(__dp4a(v.y0.y, HI, __dp4a(v.y1.y, HI, M))));
#pragma unroll
  for (int k = 0; k < 4; ++k) P[k] = __fadd2_rn(P[k], nmag);
  P[4] = make_float2(__shfl_down_sync(0xffffffffu, P[0].x, 1),
                     __shfl_down_sync(0xffffffffu, P[0].y, 1));
  P[5] = make_float2(__shfl_down_sync(0xffffffffu, P[1].x, 1),
                     __shfl_down_sync(0xffffffffu, P[1].y, 1));
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 D = __ffma2_rn(P[i], m1, P[i + 2]);
    const float2 R = __fadd2_rn(__fadd2_rn(P[i], P[i + 1]), P[i + 2]);
    const float2 gx = __fadd2_rn(d12[i], D);
    const float2 gy = __ffma2_rn(R, m1, r1[i]);
    d12[i] = __fadd2_rn(d2[i], D);
    d2[i] = D;
    r1[i] = r2[i];
    r2[i] = R;
    if constexpr (EMIT) {
      // pooled sums and their Prewitt sums are integers, so U = gx^2 + gy^2 is
      // exact below 2^24 (one rounding above) and G1 - G2 = K (U1 - U2) needs
      // no factored form; K^2 moves into the denominator's constant
      const float2 U = __ffma2_rn(gx, gx, __fmul2_rn(gy, gy));
      const float2 G = __ffma2_rn(U, kk, ee);
      const float dU = U.x - U.y;
      const float S = G.x + G.y;
      const float G12 = G.x * G.y;
      float d = -__fdividef(dU * dU, (S + 2.f * G12 * rsqrtf(G12)) * fmaf(S, KI2, TK));
      d = i < ncol ? d : 0.f;
      fs += d;
      fs2 = fmaf(d, d, fs2);
    }
  }
}

__global__ void __launch_bounds__(GR_T, GR_PER_SM) gmsd_reg_kernel(const GmsdArgs p) {
  __shared__ double s_red[2][GR_WARPS];
  __shared__ int s_flag;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int plane = blockIdx.z;
  const int pn = plane / p.Cm, pc = plane - pn * p.Cm;
  const int strip = blockIdx.x * GR_WARPS + wid;
  const int j0 = strip * GR_OW;  // first map (and pooled) column of the strip
  const int r0 = blockIdx.y * p.RH;
  const int rows = min(p.RH, p.Hout - r0);
  float fs = 0.f, fs2 = 0.f;
  if (j0 < p.Wout && rows > 0) {  // uniform per warp
    // W is a multiple of 8: a lane's 8 bytes are all inside the row or all
    // past it; a lane past it reads the row's first word (never emitted)
    const int cb = 2 * (j0 + 4 * lane);
    const long long off = (long long)pn * p.sn + (long long)pc * p.sc +
                          (long long)(2 * r0) * p.sh + (cb + 8 <= p.W ? cb : 0);
    const unsigned char* bx = reinterpret_cast<const unsigned char*>(p.x) + off;
    const unsigned char* by = reinterpret_cast<const unsigned char*>(p.y) + off;
    const long long sh = p.sh, sh2 = 2 * p.sh;
    const int np = rows + 2;  // pooled rows of the chunk (>= 3)
    auto load = [&](int g) {  // pooled row g of the chunk
      const long long o = g * sh2;
      GrRows v;
      v.x0 = __ldg(reinterpret_cast<const uint2*>(bx + o));
      v.x1 = __ldg(reinterpret_cast<const uint2*>(bx + o + sh));
      v.y0 = __ldg(reinterpret_cast<const uint2*>(by + o));
      v.y1 = __ldg(reinterpret_cast<const uint2*>(by + o + sh));
      return v;
    };
    const float2 ee = make_float2(p.eps, p.eps);
    const float TK = p.T * (144.0f * 144.0f);
    const int ncol = lane < 31 ? min(4, p.Wout - (j0 + 4 * lane)) : 0;
    float2 d2[4], d12[4], r1[4], r2[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) d2[i] = d12[i] = r1[i] = r2[i] = make_float2(0.f, 0.f);
    // two pooled rows are in flight while two earlier ones compute
    GrRows A = load(0), B = load(1);
    GrRows C = load(2), D = load(min(3, np - 1));
    gr_step<false>(A, d2, d12, r1, r2, ncol, TK, ee, fs, fs2);
    gr_step<false>(B, d2, d12, r1, r2, ncol, TK, ee, fs, fs2);
    int g = 2;  // C, D hold rows g, g + 1
#pragma unroll 1
    for (; g + 4 <= np; g += 4) {
      A = load(g + 2);
      B = load(g + 3);
      gr_step<true>(C, d2, d12, r1, r2, ncol, TK, ee, fs, fs2);
      gr_step<true>(D, d2, d12, r1, r2, ncol, TK, ee, fs, fs2);
      C = load(min(g + 4, np - 1));
      D = load(min(g + 5, np - 1));
      gr_step<true>(A, d2, d12, r1, r2, ncol, TK, ee, fs, fs2);
      gr_step<true>(B, d2, d12, r1, r2, ncol, TK, ee, fs, fs2);
    }
    if (g < np) gr_step<true>(C, d2, d12, r1, r2, ncol, TK, ee, fs, fs2);
    if (g + 1 < np) gr_step<true>(D, d2, d12, r1, r2, ncol, TK, ee, fs, fs2);
    if (g + 2 < np) gr_step<true>(load(g + 2), d2, d12, r1, r2, ncol, TK, ee, fs, fs2);
  }
  // block partials [P][bpp][2] -> last-block finalisation
  double s = warp_sum((double)fs), s2 = warp_sum((double)fs2);
  if (lane == 0) {
    s_red[0][wid] = s;
    s_red[1][wid] = s2;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double a = 0.0, b = 0.0;
    for (int w = 0; w < GR_WARPS; ++w) {
      a += s_red[0][w];
      b += s_red[1][w];
    }
    const int bpp = p.strips * p.chunks;
    const long long pidx = ((long long)plane * bpp + blockIdx.y * p.strips + blockIdx.x) * 2;
    p.part[pidx] = a;
    p.part[pidx + 1] = b;
  }
  if (last_block_arrived(p.counter, gridDim.x * gridDim.y * gridDim.z, &s_flag))
    gmsd_finalize(p, p.strips * p.chunks);
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
  // two full waves of the 3 blocks per SM gmsd_tma_kernel keeps resident,
  // each block streaming many rows
  long long want = (6LL * sms + (long long)g.strips * planes - 1) / ((long long)g.strips * planes);
  if (want < 1) want = 1;
  long long maxc = (Hout + GM_R - 1) / GM_R;
  if (want > maxc) want = maxc;
  g.RH = (int)((Hout + want - 1) / want);
  g.RH = ((g.RH + GM_R - 1) / GM_R) * GM_R;
  g.chunks = (Hout + g.RH - 1) / g.RH;
  return g;
}

// gmsd_reg_kernel: blocks of 8 strips across, chunks of rows down.  The
// chunk count minimises waves x (rows per chunk + 2 halo rows), the time a
// resident slot is busy: e.g. 192 planes of 1080p take 3 chunks (2 waves of
// 182-row blocks) rather than 1 (a third of the slots idle); chunks keep at
// least 16 rows, so a small batch does not re-read most of its rows.
static GmPlan gr_plan(int Hout, int Wout, int planes, int device) {
  GmPlan g;
  const int warps = (Wout + GR_OW - 1) / GR_OW;
  g.strips = (warps + GR_WARPS - 1) / GR_WARPS;
  const long long across = (long long)g.strips * planes;
  const long long slots = (long long)GR_PER_SM * sm_count(device);
  long long best = -1;
  g.chunks = 1;
  // at least 16 rows per chunk (at most 2/16 of the rows are halo re-reads)
  const int cmax = std::max(1, std::min((Hout + 15) / 16, 256));
  for (int c = 1; c <= cmax; ++c) {
    const int rh = (Hout + c - 1) / c;
    const long long waves = (across * c + slots - 1) / slots;
    const long long cost = waves * (rh + 2);
    if (best < 0 || cost < best) {
      best = cost;
      g.chunks = c;
    }
  }
  g.RH = (Hout + g.chunks - 1) / g.chunks;
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
  const GmPlan g = gm_plan(Ho, Wo, planes, device), r = gr_plan(Ho, Wo, planes, device);
  const size_t bpp = std::max((size_t)g.strips * g.chunks, (size_t)r.strips * r.chunks);
  return FAB_COUNTER_BYTES + 2 * sizeof(double) * (size_t)planes * bpp;
}

template <typename T, bool DOWN, bool LUMA>
static int gm_launch(GmsdArgs& p, cudaStream_t st) {
  dim3 grid(p.strips, p.chunks, p.P);
  if (p.map) gmsd_kernel<T, DOWN, LUMA, true><<<grid, GM_T, 0, st>>>(p);
  else gmsd_kernel<T, DOWN, LUMA, false><<<grid, GM_T, 0, st>>>(p);
  FAB_LAUNCH_CHECK();
  return FA_OK;
}

template <bool DOWN, bool MAP>
static int gm_launch_tma(GmsdArgs& p, int device, cudaStream_t st) {
  auto kern = gmsd_tma_kernel<DOWN, MAP>;
  static bool done[64] = {false};
  FAB_TRY(ensure_smem(kern, GmTma<DOWN>::SMEM, device, done));
  dim3 grid(p.strips, p.chunks, p.P);
  kern<<<grid, GM_T, GmTma<DOWN>::SMEM, st>>>(p);
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
  p.err = wait_error_word();
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
  // uint8, pooled, no map, rows of whole 8-byte words: the register-streaming
  // kernel
  const auto al8 = [](const View& v) {
    return reinterpret_cast<uintptr_t>(v.data) % 8 == 0 && v.sh % 8 == 0 &&
           (v.c == 1 || v.sc % 8 == 0) && (v.n == 1 || v.sn % 8 == 0);
  };
  if (dtype == FA_U8 && !luma && down && !p.map && x.w % 8 == 0 && al8(x) && al8(y)) {
    const GmPlan r = gr_plan(p.Hout, p.Wout, p.P, device);
    if (ws_bytes < FAB_COUNTER_BYTES + 2 * sizeof(double) * (size_t)p.P * r.strips * r.chunks)
      return FA_E_ARG;
    p.strips = r.strips; p.chunks = r.chunks; p.RH = r.RH;
    dim3 grid(r.strips, r.chunks, p.P);
    gmsd_reg_kernel<<<grid, GR_T, 0, st>>>(p);
    FAB_LAUNCH_CHECK();
    return FA_OK;
  }
  if (dtype == FA_U8 && !luma) {
    int dx = 0, dy = 0;
    if (make_row_map(&p.tmx, x, FA_U8, GMT_BOX, &dx) && make_row_map(&p.tmy, y, FA_U8, GMT_BOX, &dy) &&
        dx == dy) {
      p.tma_d = dx;
      if (p.map)
        return down ? gm_launch_tma<true, true>(p, device, st)
                    : gm_launch_tma<false, true>(p, device, st);
      return down ? gm_launch_tma<true, false>(p, device, st)
                  : gm_launch_tma<false, false>(p, device, st);
    }
  }
  switch (dtype) {
    case FA_U8: return gm_disp<unsigned char>(p, down, luma != nullptr, st);
    case FA_F16: return gm_disp<f16_t>(p, down, luma != nullptr, st);
    case FA_BF16: return gm_disp<bf16_t>(p, down, luma != nullptr, st);
    case FA_F32: return gm_disp<float>(p, down, luma != nullptr, st);
    case FA_F64: return gm_disp<double>(p, down, luma != nullptr, st);
    case FA_U16: return gm_disp<unsigned short>(p, down, luma != nullptr, st);
    default: return FA_E_DTYPE;
  }
}

}  // namespace fab

// ---------------------------------------------------------------------------
// Backward of GMS / GMSD (the reference differentiates its portable torch
// path, functional.py:925-971; here one fused kernel).
//   dL/dq = gm/n + gs (q - mu) / (n sigma)     per image (n map values)
//   q = (2 g1 g2 + T)/D, D = g1^2 + g2^2 + T:  dq/dg1 = 2 (g2 - q g1)/D
//   g1 = sqrt(gx1^2 + gy1^2 + eps):            dg1/dgx1 = gx1 / g1
//   gx = Prewitt_x/3 (*) pooled x  ->  d pooled = transposed Prewitt of the
//   coefficients; the 2x2 mean pool spreads 1/4 to each of its inputs.
// A block owns a 32x32 tile of pooled gradient positions: it pools the 36x36
// input region it needs into shared memory, forms the four coefficient maps
// on the 34x34 map positions that touch the tile, and gathers.
// ---------------------------------------------------------------------------
namespace fab {

constexpr int GB_T = 32;           // pooled gradient tile
constexpr int GB_C = GB_T + 2;     // coefficient positions that reach the tile
constexpr int GB_P = GB_T + 4;     // pooled values the coefficients need

struct GmsdBwdArgs {
  const float* x;
  const float* y;
  int N, C, H, W, Hd, Wd, Hout, Wout, down;
  float T, eps;
  const double* gm;   // [N] dL/d(gms per image), nullable
  const double* gsd;  // [N] dL/d(gmsd per image), nullable
  const double* mu;   // [N] forward gms
  const double* sd;   // [N] forward gmsd
  double npix;        // C * Hout * Wout
  float* dx;
  float* dy;
};

__global__ void __launch_bounds__(256) gmsd_bwd_kernel(GmsdBwdArgs p) {
  __shared__ float px[GB_P][GB_P + 1], py[GB_P][GB_P + 1];
  __shared__ float c1x[GB_C][GB_C + 1], c1y[GB_C][GB_C + 1];  // dL/dgx1, dL/dgy1
  __shared__ float c2x[GB_C][GB_C + 1], c2y[GB_C][GB_C + 1];  // dL/dgx2, dL/dgy2
  const int plane = blockIdx.z, n = plane / p.C;
  const int tr = blockIdx.y * GB_T, tc = blockIdx.x * GB_T;  // first pooled row/col of the tile
  const long long pbase = (long long)plane * p.H * p.W;
  const int tid = threadIdx.x;
  // 1. pooled inputs on rows tr-2 .. tr+33, cols tc-2 .. tc+33 (zero outside)
  for (int i = tid; i < GB_P * GB_P; i += 256) {
    const int r = i / GB_P, c = i - r * GB_P;
    const int pr = tr - 2 + r, pc = tc - 2 + c;
    float a = 0.f, b = 0.f;
    if (pr >= 0 && pr < p.Hd && pc >= 0 && pc < p.Wd) {
      if (p.down) {
        const long long o = pbase + (long long)(2 * pr) * p.W + 2 * pc;
        a = 0.25f * (__ldg(p.x + o) + __ldg(p.x + o + 1) + __ldg(p.x + o + p.W) + __ldg(p.x + o + p.W + 1));
        b = 0.25f * (__ldg(p.y + o) + __ldg(p.y + o + 1) + __ldg(p.y + o + p.W) + __ldg(p.y + o + p.W + 1));
      } else {
        const long long o = pbase + (long long)pr * p.W + pc;
        a = __ldg(p.x + o);
        b = __ldg(p.y + o);
      }
    }
    px[r][c] = a;
    py[r][c] = b;
  }
  __syncthreads();
  // 2. coefficients at map positions tr-2 .. tr+31 (zero outside the map)
  const double gm = p.gm ? p.gm[n] : 0.0, gs = p.gsd ? p.gsd[n] : 0.0;
  const double sdn = p.sd[n];
  const float alpha = (float)(gm / p.npix - (sdn > 0.0 ? gs * p.mu[n] / (p.npix * sdn) : 0.0));
  const float beta = (float)(sdn > 0.0 ? gs / (p.npix * sdn) : 0.0);
  constexpr float THIRD = 1.0f / 3.0f;
  for (int i = tid; i < GB_C * GB_C; i += 256) {
    const int r = i / GB_C, c = i - r * GB_C;
    const int mr = tr - 2 + r, mc = tc - 2 + c;
    float ax = 0.f, ay = 0.f, bx = 0.f, by = 0.f;
    if (mr >= 0 && mr < p.Hout && mc >= 0 && mc < p.Wout) {
      const float gx1 = ((px[r][c] - px[r][c + 2]) + (px[r + 1][c] - px[r + 1][c + 2]) +
                         (px[r + 2][c] - px[r + 2][c + 2])) * THIRD;
      const float gy1 = ((px[r][c] - px[r + 2][c]) + (px[r][c + 1] - px[r + 2][c + 1]) +
                         (px[r][c + 2] - px[r + 2][c + 2])) * THIRD;
      const float gx2 = ((py[r][c] - py[r][c + 2]) + (py[r + 1][c] - py[r + 1][c + 2]) +
                         (py[r + 2][c] - py[r + 2][c + 2])) * THIRD;
      const float gy2 = ((py[r][c] - py[r + 2][c]) + (py[r][c + 1] - py[r + 2][c + 1]) +
                         (py[r][c + 2] - py[r + 2][c + 2])) * THIRD;
      const float g1 = sqrtf(fmaf(gx1, gx1, fmaf(gy1, gy1, p.eps)));
      const float g2 = sqrtf(fmaf(gx2, gx2, fmaf(gy2, gy2, p.eps)));
      const float D = fmaf(g1, g1, fmaf(g2, g2, p.T));
      const float q = fmaf(2.f * g1, g2, p.T) / D;
      const float up = fmaf(beta, q, alpha);           // dL/dq
      const float k1 = up * 2.f * (g2 - q * g1) / (D * g1);  // dL/dg1 / g1
      const float k2 = up * 2.f * (g1 - q * g2) / (D * g2);
      ax = k1 * gx1; ay = k1 * gy1; bx = k2 * gx2; by = k2 * gy2;
    }
    c1x[r][c] = ax; c1y[r][c] = ay; c2x[r][c] = bx; c2y[r][c] = by;
  }
  __syncthreads();
  // 3. transposed Prewitt: pooled (i, j) gathers map positions (i-a, j-b)
  for (int i = tid; i < GB_T * GB_T; i += 256) {
    const int r = i / GB_T, c = i - r * GB_T;
    const int pr = tr + r, pc = tc + c;
    if (pr >= p.Hd || pc >= p.Wd) continue;
    float sx = 0.f, sy = 0.f;
#pragma unroll
    for (int a = 0; a < 3; ++a) {
#pragma unroll
      for (int b = 0; b < 3; ++b) {
        const int cr = r + 2 - a, cc = c + 2 - b;   // map position (pr - a, pc - b)
        const float kx = (b == 0) ? THIRD : (b == 2 ? -THIRD : 0.f);
        const float ky = (a == 0) ? THIRD : (a == 2 ? -THIRD : 0.f);
        sx = fmaf(kx, c1x[cr][cc], fmaf(ky, c1y[cr][cc], sx));
        sy = fmaf(kx, c2x[cr][cc], fmaf(ky, c2y[cr][cc], sy));
      }
    }
    if (p.down) {
      const long long o = pbase + (long long)(2 * pr) * p.W + 2 * pc;
      const float gx = 0.25f * sx, gy = 0.25f * sy;
      if (p.dx) { p.dx[o] = gx; p.dx[o + 1] = gx; p.dx[o + p.W] = gx; p.dx[o + p.W + 1] = gx; }
      if (p.dy) { p.dy[o] = gy; p.dy[o + 1] = gy; p.dy[o + p.W] = gy; p.dy[o + p.W + 1] = gy; }
    } else {
      const long long o = pbase + (long long)pr * p.W + pc;
      if (p.dx) p.dx[o] = sx;
      if (p.dy) p.dy[o] = sy;
    }
  }
}

int gmsd_backward_impl(const float* x, const float* y, int N, int C, int H, int W, int down,
                       double T, double eps, const double* gm, const double* gsd,
                       const double* mu, const double* sd, float* dx, float* dy, int device,
                       cudaStream_t st) {
  (void)device;
  if (!x || !y || !mu || !sd || (!dx && !dy) || (!gm && !gsd)) return FA_E_ARG;
  if (N <= 0 || C <= 0 || H <= 0 || W <= 0) return FA_E_SHAPE;
  GmsdBwdArgs p{};
  if (!gm_dims(H, W, down, &p.Hd, &p.Wd, &p.Hout, &p.Wout)) return FA_E_SHAPE;
  if ((long long)N * C > 65535) return FA_E_SHAPE;
  p.x = x; p.y = y; p.N = N; p.C = C; p.H = H; p.W = W; p.down = down ? 1 : 0;
  p.T = (float)T; p.eps = (float)eps;
  p.gm = gm; p.gsd = gsd; p.mu = mu; p.sd = sd;
  p.npix = (double)C * p.Hout * p.Wout;
  p.dx = dx; p.dy = dy;
  dim3 grid((p.Wd + GB_T - 1) / GB_T, (p.Hd + GB_T - 1) / GB_T, N * C);
  gmsd_bwd_kernel<<<grid, 256, 0, st>>>(p);
  FAB_LAUNCH_CHECK();
  return FA_OK;
}

}  // namespace fab
