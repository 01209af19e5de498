// Fused SSIM backward on sm_100a: one launch, no frame-sized scratch.
//
// Replaces the reference's two-kernel backward (MODE_PREP / MODE_PREP_CS of
// ssim_fused_kernel, fa_cuda.cu:551-607, writing 3-4 coefficient planes to
// global memory, then ssim_bwd_scatter_kernel, fa_cuda.cu:655-784, reading
// them back).  For an output position o with upstream gradient g:
//   b = g dS/dsxx, c = g dS/dsxy, t_x = g dS/dmx - 2 b ux - c uy
//   (MS-SSIM: b = -(gS S + gCS cs)/B2, c = 2 (gS A1/B1 + gCS)/B2)
//   dx(i) = 2 x'(i) (w*b)(i) + y'(i) (w*c)(i) + (w*t_x)(i)     (w* transposed)
// and symmetrically for dy.  Here one block streams a strip of rows through
// moments -> coefficients (shared memory) -> transposed blur -> dx/dy, so the
// coefficients never leave the SM.  A strip of 32*KW moment columns yields
// 32*KW - (KW-1) gradient columns.
//
// Fused forward mode (FWD): for a scalar loss the gradient is linear in the
// upstream scalar, so the same pass can return the SSIM means (each moment
// position summed by the one block that owns it: columns [c0, c0 + TD), rows
// [r0, r0 + rows)) together with the gradient of the batch-mean SSIM for an
// upstream gradient of 1.  A training step then needs no separate forward
// launch; the caller scales the unit gradient when the real upstream
// gradient arrives.
#include <type_traits>

#include "ssim_common.cuh"

namespace fab {

constexpr int G_MAP = 0;     // dL/dmap per position
constexpr int G_SCALAR = 1;  // dL/d(batch mean), one device scalar
constexpr int G_PLANE = 2;   // dL/d(plane-mean S) and dL/d(plane-mean cs)

template <int KW>
struct BwdGeo {
  using G = Geo<KW>;
  using R = Raw<float, KW>;
  static constexpr int SCW = (G::NT + KW - 1 + 7) / 8 * 8;  // coefficient row width, zero padded
  static constexpr size_t kH = sizeof(float4) * KW * G::NT;
  static constexpr size_t kC = sizeof(float4) * KW * SCW;
  static constexpr size_t kX = R::kFloatBytes;  // staged moment rows, x and y
  static constexpr size_t kD = R::kFloatBytes;  // x and y at the gradient rows
  static constexpr size_t kBytes = kH + kC + kX + kD;
  static_assert(kH % 128 == 0 && kC % 128 == 0, "TMA destinations must stay aligned");
};

// floor division for the (possibly negative) strip origin
__device__ __forceinline__ int floor_to(int v, int a) {
  return (v >= 0 ? v / a : -((-v + a - 1) / a)) * a;
}

// STAGE_TMA: TMA staging (row pitch a multiple of 16 bytes); STAGE_GENERIC:
// register staging and direct loads for any float32 rows (built with both
// gradients only; a null dx or dy is simply not written).
template <int KW, bool DX, bool DY, int GMODE, int STAGE, bool FWD>
__global__ void __launch_bounds__(32 * KW, 1) ssim_bwd_kernel(const __grid_constant__ SsimArgs p) {
  constexpr bool TMA = (STAGE == STAGE_TMA);
  using G = Geo<KW>;
  using B = BwdGeo<KW>;
  constexpr int NPL = (DX && DY) ? 4 : 3;
  using R = Raw<float, KW>;
  extern __shared__ __align__(128) float4 smem4[];
  float4* sH = smem4;                                 // [KW][NT] moments, then scatter rows
  float4* sC = sH + KW * G::NT;                       // [KW][SCW] coefficients
  float* sX = reinterpret_cast<float*>(sC + KW * B::SCW);  // [KW][RP] staged inputs
  float* sY = sX + KW * R::RP;
  float* dX = sY + KW * R::RP;                        // [KW][RP] x at the gradient rows
  float* dY = dX + KW * R::RP;
  __shared__ __align__(8) unsigned long long s_bar[2];  // staging, gradient rows
  __shared__ double s_red[32];
  __shared__ int s_flag;

  const int t = threadIdx.x;
  const int lane = t & 31, warp = t >> 5;
  const int plane = blockIdx.z;
  const int pn = plane / p.C, pc = plane - pn * p.C;
  const long long pbase = (long long)plane * p.H * p.W;
  const int c0 = blockIdx.x * G::TD;      // first gradient column of the strip
  const int mc0 = c0 - (KW - 1);          // first moment column
  const int r0 = blockIdx.y * p.RH;       // first gradient row of the chunk
  const int rows = min(p.RH, p.H - r0);
  const int i0 = r0 - (KW - 1);           // first input row
  const int iters = (rows + 2 * (KW - 1) + KW - 1) / KW;
  const int q = mc0 + t;                  // this thread's moment column
  const bool q_ok = q >= 0 && q < p.Wout;
  const int dcol = c0 + t;                // this thread's gradient column
  const bool d_ok = t < G::TD && dcol < p.W;
  // TMA x coordinates rounded down to 16 bytes, and the offsets into the rows
  const int xs0 = floor_to(mc0 + p.tma_d, R::XA), sofs = mc0 + p.tma_d - xs0;
  const int xd0 = floor_to(c0 + p.tma_d, R::XA), dofs = c0 + p.tma_d - xd0;

  // zero the coefficient padding columns once
  for (int i = t; i < KW * (B::SCW - G::NT); i += G::NT) {
    const int r = i / (B::SCW - G::NT), c = i - r * (B::SCW - G::NT);
    sC[r * B::SCW + G::NT + c] = make_float4(0.f, 0.f, 0.f, 0.f);
  }

  float gS = 0.f, gCS = 0.f;
  if (GMODE == G_SCALAR) gS = (FWD ? 1.f : __ldg(p.gscalar)) * p.grad_norm;
  const bool own_col = q_ok && t >= KW - 1;  // moment column q lies in [c0, c0 + TD)
  double acc_s = 0.0;
  if (GMODE == G_PLANE) {
    gS = __ldg(p.gs + plane) * p.grad_norm;
    gCS = __ldg(p.gcs + plane) * p.grad_norm;
  }

  float vx[TMA ? 1 : G::NE], vy[TMA ? 1 : G::NE];
  if constexpr (TMA) {
    if (t == 0) {
      mbar_init(&s_bar[0], 1);
      mbar_init(&s_bar[1], 1);
    }
    fence_async_smem();
    __syncthreads();
    stage_tma<float, KW>(p, pn, pc, i0, xs0, sX, sY, &s_bar[0]);
  } else {
    stage_load<float, false, KW>(p, pbase, i0, mc0, vx, vy);
    stage_store<KW, R::RP>(sX, sY, vx, vy);
  }
  const int so = TMA ? sofs : 0;

  float4 ring1[KW], ring2[KW];
#pragma unroll
  for (int k = 0; k < KW; ++k) {
    ring1[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    ring2[k] = make_float4(0.f, 0.f, 0.f, 0.f);
  }

  for (int m = 0; m < iters; ++m) {
    if constexpr (TMA) {
      mbar_wait(&s_bar[0], m & 1);
      stage_convert<float, KW>(p, sX, sY, sX, sY);
    }
    __syncthreads();
    // the input values at this iteration's gradient rows (L2-resident)
    if constexpr (TMA)
      stage_tma<float, KW>(p, pn, pc, i0 + m * KW - (KW - 1), xd0, dX, dY, &s_bar[1]);
    // horizontal moments: warp k -> staged row k
    {
      const float* rx = sX + warp * R::RP + so + lane * KW;
      const float* ry = sY + warp * R::RP + so + lane * KW;
      float4* out = sH + warp * G::NT + lane * KW;
      hblur_xy<KW>(p, rx, ry, out);
      hblur_prod<KW>(p, rx, ry, out);
    }
    __syncthreads();
    const bool more = (m + 1 < iters);
    if (more) {
      if constexpr (TMA) stage_tma<float, KW>(p, pn, pc, i0 + (m + 1) * KW, xs0, sX, sY, &s_bar[0]);
      else stage_load<float, false, KW>(p, pbase, i0 + (m + 1) * KW, mc0, vx, vy);
    }
    // vertical moments -> coefficients
    float fs = 0.f;
#pragma unroll
    for (int k = 0; k < KW; ++k) {
      ring1[k] = sH[k * G::NT + t];
      const int L = m * KW + k;
      const int o = i0 + L - (KW - 1);  // moment row
      float4 cf = make_float4(0.f, 0.f, 0.f, 0.f);
      if (L >= KW - 1 && o >= 0 && o < p.Hout && q_ok) {
        const Moments mo = moments(p, vblur_at<KW, 4>(p, ring1, k));
        // one reciprocal: 1/B1 = B2/(B1 B2), 1/B2 = B1/(B1 B2)
        const float inv = 1.0f / (mo.B1 * mo.B2);
        const float iB1 = mo.B2 * inv;
        const float iB2 = mo.B1 * inv;
        const float S = mo.A1 * mo.A2 * inv;
        const float kk = 2.f * mo.A2 * inv;
        if (FWD && own_col && o >= r0 && o < r0 + rows) fs += S;
        float g = gS, bb, cc;
        if (GMODE == G_MAP)
          g = __ldg(p.dmap + (long long)plane * p.Hout * p.Wout + (long long)o * p.Wout + q);
        if (GMODE == G_PLANE) {
          const float CS = mo.A2 * iB2;
          bb = -(g * S + gCS * CS) * iB2;
          cc = 2.f * (g * mo.A1 * iB1 + gCS) * iB2;
        } else {
          bb = -g * S * iB2;
          cc = 2.f * g * mo.A1 * inv;
        }
        cf.x = bb;
        cf.y = cc;
        if (DX) cf.z = g * kk * (mo.my - mo.mx * mo.A1 * iB1) - 2.f * bb * mo.ux - cc * mo.uy;
        if (DY) {
          const float ty = g * kk * (mo.mx - mo.my * mo.A1 * iB1) - 2.f * bb * mo.uy - cc * mo.ux;
          if (DX) cf.w = ty;
          else cf.z = ty;
        }
      }
      sC[k * B::SCW + t] = cf;
    }
    if constexpr (FWD) acc_s += (double)fs;
    __syncthreads();
    // horizontal scatter of the coefficient rows
    {
      const float4* rc = sC + warp * B::SCW + lane * KW;
      float4* out = sH + warp * G::NT + lane * KW;
      hblur_pair<KW, 0, 2, false, true>(p, rc, out);  // reversed window: adjoint
      hblur_pair<KW, 1, NPL - 2, false, true>(p, rc, out);
    }
    if constexpr (TMA) mbar_wait(&s_bar[1], m & 1);
    __syncthreads();
    // vertical scatter -> dx, dy
#pragma unroll
    for (int k = 0; k < KW; ++k) {
      ring2[k] = sH[k * G::NT + t];
      const int L = m * KW + k;
      const int r = i0 + L - (KW - 1);  // gradient row
      if (L >= 2 * (KW - 1) && r < r0 + rows && d_ok) {
        const float4 s = vblur_at<KW, NPL, false, true>(p, ring2, k);
        const long long off = (long long)r * p.W + dcol;
        float xs, ys;
        if constexpr (TMA) {
          xs = dX[k * R::RP + dofs + t] - p.shift;
          ys = dY[k * R::RP + dofs + t] - p.shift;
        } else {
          xs = __ldg(reinterpret_cast<const float*>(p.x) + pbase + off) - p.shift;
          ys = __ldg(reinterpret_cast<const float*>(p.y) + pbase + off) - p.shift;
        }
        if (DX && p.dx) p.dx[pbase + off] = fmaf(2.f * xs, s.x, fmaf(ys, s.y, s.z));
        if (DY && p.dy) p.dy[pbase + off] = fmaf(2.f * ys, s.x, fmaf(xs, s.y, (DX && DY) ? s.w : s.z));
      }
    }
    if constexpr (!TMA) {
      if (more) {
        __syncthreads();  // every h1 read of this iteration's rows is long done; keep it simple
        stage_store<KW, R::RP>(sX, sY, vx, vy);
      }
    }
  }
  if constexpr (FWD) {
    const int bpp = p.strips * p.chunks;
    acc_s = block_sum(acc_s, s_red);
    if (t == 0) p.part_s[(long long)plane * bpp + blockIdx.y * p.strips + blockIdx.x] = acc_s;
    if (last_block_arrived(p.counter, gridDim.x * gridDim.y * gridDim.z, &s_flag))
      ssim_fwd_finalize(p, bpp);
  }
}

// ---------------------------------------------------------------------------
// Warp-specialised form (TMA staging).  Two groups of 32*KW threads run in
// lockstep, two phases per batch of KW rows, separated by block barriers:
//   group A (moments):  phase 1  horizontal moments of batch m -> sH
//                       phase 2  issue the copy of batch m+1; vertical moments
//                                and coefficients of batch m -> sC
//   group B (scatter):  phase 1  horizontal scatter of batch m-1 (sC -> sS)
//                       phase 2  vertical scatter of batch m-1 -> dx / dy
// Each thread keeps one register ring instead of both, so twice the warps fit
// on an SM, and each group's work fills the other's barrier tails.  The
// staged rows are read raw (the shift is applied as they are loaded), and the
// inputs at the gradient rows come from L2, read two batches after staging.
// ---------------------------------------------------------------------------
template <int KW>
struct WsGeo {
  using G = Geo<KW>;
  using B = BwdGeo<KW>;
  using R = Raw<float, KW>;
  static constexpr size_t kH = sizeof(float4) * KW * G::NT;
  static constexpr size_t kC = sizeof(float4) * KW * B::SCW;
  static constexpr size_t kS = sizeof(float4) * KW * G::NT;
  static constexpr size_t kX = sizeof(float) * 2 * KW * R::RP;
  static constexpr size_t kBytes = kH + kC + kS + kX;
  static_assert(kBytes <= 227 * 1024, "shared memory budget");
};

// Horizontal blurs of the warp-specialised kernel, symmetric taps.  Each
// thread's KW outputs are produced in three passes (outputs [O0, O0 + NO)) so
// that only NO accumulator pairs are live next to the thread's register
// ring; the passes re-read KW - 1 staged inputs.
template <int KW, int O0, int NO>
__device__ __forceinline__ void hblur_raw_part(const SsimArgs& p, const float* __restrict__ sx,
                                               const float* __restrict__ sy,
                                               float4* __restrict__ out) {
  const float2 nsh = make_float2(-p.shift, -p.shift);
  float2 a[NO], b[NO];
#pragma unroll
  for (int o = 0; o < NO; ++o) a[o] = b[o] = make_float2(0.f, 0.f);
#pragma unroll
  for (int q = O0; q < O0 + NO + KW - 1; ++q) {
    const float2 c = __fadd2_rn(make_float2(sx[q], sy[q]), nsh);  // shifted x', y'
    const float dv = c.x - c.y;  // from the shifted values, as the forward kernel forms it
    const float2 v = make_float2(c.x * c.y, dv * dv);  // x'y', (x'-y')^2
#pragma unroll
    for (int o = 0; o < NO; ++o) {
      const int j = q - (O0 + o);
      if (j >= 0 && j < KW) {
        const float2 w = p.w2[tap<KW, true>(j)];
        a[o] = __ffma2_rn(w, c, a[o]);
        b[o] = __ffma2_rn(w, v, b[o]);
      }
    }
  }
#pragma unroll
  for (int o = 0; o < NO; ++o) out[O0 + o] = make_float4(a[o].x, a[o].y, b[o].x, b[o].y);
}

template <int KW>
__device__ __forceinline__ void hblur_raw(const SsimArgs& p, const float* sx, const float* sy,
                                          float4* out) {
  constexpr int H = (KW + 2) / 3;  // three passes
  hblur_raw_part<KW, 0, H>(p, sx, sy, out);
  hblur_raw_part<KW, H, H>(p, sx, sy, out);
  hblur_raw_part<KW, 2 * H, KW - 2 * H>(p, sx, sy, out);
}

// Scatter rows: NC (3 or 4) coefficient components, outputs [O0, O0 + NO).
template <int KW, int NC, int O0, int NO>
__device__ __forceinline__ void hscatter_part(const SsimArgs& p, const float4* __restrict__ sc,
                                              float4* __restrict__ out) {
  float2 a[NO], b[NO];
#pragma unroll
  for (int o = 0; o < NO; ++o) a[o] = b[o] = make_float2(0.f, 0.f);
#pragma unroll
  for (int q = O0; q < O0 + NO + KW - 1; ++q) {
    const float4 v = sc[q];
#pragma unroll
    for (int o = 0; o < NO; ++o) {
      const int j = q - (O0 + o);
      if (j >= 0 && j < KW) {
        const float2 w = p.w2[tap<KW, true>(j)];
        a[o] = __ffma2_rn(w, make_float2(v.x, v.y), a[o]);
        if (NC == 4) b[o] = __ffma2_rn(w, make_float2(v.z, v.w), b[o]);
        else b[o].x = fmaf(w.x, v.z, b[o].x);
      }
    }
  }
#pragma unroll
  for (int o = 0; o < NO; ++o) out[O0 + o] = make_float4(a[o].x, a[o].y, b[o].x, b[o].y);
}

template <int KW, int NC>
__device__ __forceinline__ void hscatter(const SsimArgs& p, const float4* sc, float4* out) {
  constexpr int H = (KW + 2) / 3;  // three passes
  hscatter_part<KW, NC, 0, H>(p, sc, out);
  hscatter_part<KW, NC, H, H>(p, sc, out);
  hscatter_part<KW, NC, 2 * H, KW - 2 * H>(p, sc, out);
}

template <int KW, int GMODE, bool FWD>
__global__ void __maxnreg__(80) ssim_bwd_ws_kernel(const __grid_constant__ SsimArgs p) {
  using G = Geo<KW>;
  using B = BwdGeo<KW>;
  using R = Raw<float, KW>;
  constexpr int NT = G::NT;
  extern __shared__ __align__(128) float4 smem4[];
  float4* sH = smem4;                                      // [KW][NT] horizontal moments
  float4* sC = sH + KW * NT;                               // [KW][SCW] coefficients
  float4* sS = sC + KW * B::SCW;                           // [KW][NT] horizontal scatter
  float* sX = reinterpret_cast<float*>(sS + KW * NT);      // [KW][RP] raw x rows
  float* sY = sX + KW * R::RP;                             // [KW][RP] raw y rows
  __shared__ __align__(8) unsigned long long s_bar;
  __shared__ double s_red[32];
  __shared__ int s_flag;

  const bool grpA = threadIdx.x < NT;
  const int t = grpA ? threadIdx.x : threadIdx.x - NT;  // column slot within the group
  const int lane = t & 31, warp = t >> 5;
  const int plane = blockIdx.z;
  const int pn = plane / p.C, pc = plane - pn * p.C;
  const long long pbase = (long long)plane * p.H * p.W;
  const int c0 = blockIdx.x * G::TD;
  const int mc0 = c0 - (KW - 1);
  const int r0 = blockIdx.y * p.RH;
  const int rows = min(p.RH, p.H - r0);
  const int i0 = r0 - (KW - 1);
  const int iters = (rows + 2 * (KW - 1) + KW - 1) / KW;
  const int xs0 = floor_to(mc0 + p.tma_d, R::XA), sofs = mc0 + p.tma_d - xs0;

  // zero the coefficient padding columns once
  for (int i = threadIdx.x; i < KW * (B::SCW - NT); i += 2 * NT) {
    const int r = i / (B::SCW - NT), c = i - r * (B::SCW - NT);
    sC[r * B::SCW + NT + c] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if (threadIdx.x == 0) mbar_init(&s_bar, 1);
  fence_async_smem();
  __syncthreads();
  stage_tma<float, KW>(p, pn, pc, i0, xs0, sX, sY, &s_bar);

  float4 ring[KW];
#pragma unroll
  for (int k = 0; k < KW; ++k) ring[k] = make_float4(0.f, 0.f, 0.f, 0.f);
  double acc_s = 0.0;  // owned SSIM values: float per batch, double across batches

  if (grpA) {
    // ---------------- group A: moments -> coefficients ----------------
    const int q = mc0 + t;
    const bool q_ok = q >= 0 && q < p.Wout;
    const bool own_col = q_ok && t >= KW - 1;
    float gS = 0.f, gCS = 0.f;
    if (GMODE == G_SCALAR) gS = (FWD ? 1.f : __ldg(p.gscalar)) * p.grad_norm;
    if (GMODE == G_PLANE) {
      gS = __ldg(p.gs + plane) * p.grad_norm;
      gCS = __ldg(p.gcs + plane) * p.grad_norm;
    }
    for (int m = 0; m <= iters; ++m) {
      if (m < iters) {
        mbar_wait(&s_bar, m & 1);
        hblur_raw<KW>(p, sX + warp * R::RP + sofs + lane * KW, sY + warp * R::RP + sofs + lane * KW,
                      sH + warp * NT + lane * KW);
      }
      __syncthreads();
      if (m < iters) {
        if (m + 1 < iters) stage_tma<float, KW>(p, pn, pc, i0 + (m + 1) * KW, xs0, sX, sY, &s_bar);
        const int o0 = i0 + m * KW - (KW - 1);  // moment row of slot 0
        float fs = 0.f;
        // CHK: per-row tests; interior batches (every row a valid, owned
        // moment row) skip them
        auto rows_step = [&](auto chk) {
          constexpr bool CHK = decltype(chk)::value;
#pragma unroll
          for (int k = 0; k < KW; ++k) {
            ring[k] = sH[k * NT + t];
            const int o = o0 + k;
            float4 cf = make_float4(0.f, 0.f, 0.f, 0.f);
            if (q_ok && (!CHK || (m * KW + k >= KW - 1 && o >= 0 && o < p.Hout))) {
              const Moments mo = moments(p, vblur_at<KW, 4, true>(p, ring, k));
              // one approximate reciprocal (a few ulp) serves S, cs and the
              // coefficients
              const float inv = __fdividef(1.0f, mo.B1 * mo.B2);
              const float iB1 = mo.B2 * inv;
              const float iB2 = mo.B1 * inv;
              const float S = mo.A1 * mo.A2 * inv;
              const float kk = 2.f * mo.A2 * inv;
              if (FWD && own_col && (!CHK || (o >= r0 && o < r0 + rows))) fs += S;
              float g = gS, bb, cc;
              if (GMODE == G_MAP)
                g = __ldg(p.dmap + (long long)plane * p.Hout * p.Wout + (long long)o * p.Wout + q);
              if (GMODE == G_PLANE) {
                const float CS = mo.A2 * iB2;
                bb = -(g * S + gCS * CS) * iB2;
                cc = 2.f * (g * mo.A1 * iB1 + gCS) * iB2;
              } else {
                bb = -g * S * iB2;
                cc = 2.f * g * mo.A1 * inv;
              }
              cf.x = bb;
              cf.y = cc;
              // both first-moment terms, whichever gradients are stored: the
              // uniform four-component layout compiles without spills
              cf.z = g * kk * (mo.my - mo.mx * mo.A1 * iB1) - 2.f * bb * mo.ux - cc * mo.uy;
              cf.w = g * kk * (mo.mx - mo.my * mo.A1 * iB1) - 2.f * bb * mo.uy - cc * mo.ux;
            }
            sC[k * B::SCW + t] = cf;
          }
        };
        const bool interior = m >= 1 && o0 >= 0 && o0 + KW - 1 < p.Hout &&
                              (!FWD || (o0 >= r0 && o0 + KW - 1 < r0 + rows));
        if (interior) rows_step(std::false_type{});
        else rows_step(std::true_type{});
        if constexpr (FWD) acc_s += (double)fs;
      }
      __syncthreads();
    }
  } else {
    // ---------------- group B: scatter -> dx / dy (one batch behind) ----------------
    const int dcol = c0 + t;
    const bool d_ok = t < G::TD && dcol < p.W;
    const float* X = reinterpret_cast<const float*>(p.x);
    const float* Y = reinterpret_cast<const float*>(p.y);
    for (int m = 0; m <= iters; ++m) {
      if (m >= 1) {
        const float4* rc = sC + warp * B::SCW + lane * KW;
        float4* out = sS + warp * NT + lane * KW;
        hscatter<KW, 4>(p, rc, out);  // packed pairs even with 3 components
      }
      __syncthreads();
      if (m >= 1) {
        const int rb = i0 + (m - 1) * KW - (KW - 1);  // gradient row of slot 0
        const long long off0 = pbase + (long long)rb * p.W + dcol;
        auto rows_step = [&](auto chk) {
          constexpr bool CHK = decltype(chk)::value;
#pragma unroll
          for (int k = 0; k < KW; ++k) {
            ring[k] = sS[k * NT + t];
            if (d_ok && (!CHK || ((m - 1) * KW + k >= 2 * (KW - 1) && rb + k < r0 + rows))) {
              const float4 sv = vblur_at<KW, 4, true>(p, ring, k);
              const long long off = off0 + (long long)k * p.W;
              const float xs = __ldg(X + off) - p.shift;
              const float ys = __ldg(Y + off) - p.shift;
              if (p.dx) p.dx[off] = fmaf(2.f * xs, sv.x, fmaf(ys, sv.y, sv.z));
              if (p.dy) p.dy[off] = fmaf(2.f * ys, sv.x, fmaf(xs, sv.y, sv.w));
            }
          }
        };
        const bool interior = (m - 1) * KW >= 2 * (KW - 1) && rb + KW - 1 < r0 + rows;
        if (interior) rows_step(std::false_type{});
        else rows_step(std::true_type{});
      }
      __syncthreads();
    }
  }
  if constexpr (FWD) {
    const int bpp = p.strips * p.chunks;
    acc_s = block_sum(acc_s, s_red);
    if (threadIdx.x == 0) p.part_s[(long long)plane * bpp + blockIdx.y * p.strips + blockIdx.x] = acc_s;
    if (last_block_arrived(p.counter, gridDim.x * gridDim.y * gridDim.z, &s_flag))
      ssim_fwd_finalize(p, bpp);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

template <int KW, bool DX, bool DY, int GMODE, int STAGE, bool FWD>
static int launch_bwd(const SsimArgs& p, int device, cudaStream_t st) {
  dim3 grid(p.strips, p.chunks, p.P);
  if (STAGE == STAGE_TMA && p.sym) {
    // one instantiation serves dx, dy or both: stores test the pointers
    auto kern = ssim_bwd_ws_kernel<KW, GMODE, FWD>;
    const size_t sm = WsGeo<KW>::kBytes;
    static bool done[64] = {false};
    FAB_TRY(ensure_smem(kern, sm, device, done));
    kern<<<grid, 64 * KW, sm, st>>>(p);
  } else {
    auto kern = ssim_bwd_kernel<KW, DX, DY, GMODE, STAGE, FWD>;
    const size_t sm = BwdGeo<KW>::kBytes;
    static bool done[64] = {false};
    FAB_TRY(ensure_smem(kern, sm, device, done));
    kern<<<grid, 32 * KW, sm, st>>>(p);
  }
  FAB_LAUNCH_CHECK();
  return FA_OK;
}

template <bool DX, bool DY, int GMODE, int STAGE, bool FWD>
static int bwd_k(const SsimArgs& p, int K, int device, cudaStream_t st) {
  switch (K) {
    case 11: return launch_bwd<11, DX, DY, GMODE, STAGE, FWD>(p, device, st);
    case 9: return launch_bwd<9, DX, DY, GMODE, STAGE, FWD>(p, device, st);
    case 7: return launch_bwd<7, DX, DY, GMODE, STAGE, FWD>(p, device, st);
    case 5: return launch_bwd<5, DX, DY, GMODE, STAGE, FWD>(p, device, st);
    case 3: return launch_bwd<3, DX, DY, GMODE, STAGE, FWD>(p, device, st);
    default: return FA_E_WINDOW;
  }
}

template <int GMODE, bool FWD = false>
static int bwd_g(const SsimArgs& p, bool tma, int K, int device, cudaStream_t st) {
  if (!tma) return bwd_k<true, true, GMODE, STAGE_GENERIC, FWD>(p, K, device, st);
  if (p.dx && p.dy) return bwd_k<true, true, GMODE, STAGE_TMA, FWD>(p, K, device, st);
  if (p.dx) return bwd_k<true, false, GMODE, STAGE_TMA, FWD>(p, K, device, st);
  return bwd_k<false, true, GMODE, STAGE_TMA, FWD>(p, K, device, st);
}

static int bwd_box_width(int K) {
  switch (K) {
    case 11: return Raw<float, 11>::BW;
    case 9: return Raw<float, 9>::BW;
    case 7: return Raw<float, 7>::BW;
    case 5: return Raw<float, 5>::BW;
    default: return Raw<float, 3>::BW;
  }
}

// Fills the launch arguments shared by the backward and the fused mode.
static int bwd_setup(SsimArgs& p, bool& tma, const float* x, const float* y, int N, int C, int H,
                     int W, const float* taps, int K, double shift, double C1, double C2,
                     float* dx, float* dy, int device) {
  if (!x || !y || !taps) return FA_E_ARG;
  if (!dx && !dy) return FA_E_ARG;
  if (N <= 0 || C <= 0 || H <= 0 || W <= 0) return FA_E_SHAPE;
  if (K < 3 || K > FA_MAX_WIN || (K & 1) == 0) return FA_E_WINDOW;
  const int Hout = H - K + 1, Wout = W - K + 1;
  if (Hout <= 0 || Wout <= 0) return FA_E_SHAPE;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 3u) return FA_E_ARG;
  p = SsimArgs{};
  p.x = reinterpret_cast<const char*>(x);
  p.y = reinterpret_cast<const char*>(y);
  p.N = N; p.C = C; p.H = H; p.W = W;
  p.Cm = C; p.P = N * C;
  if (p.P > 65535) return FA_E_SHAPE;
  p.sn = (long long)C * H * W; p.sc = (long long)H * W; p.sh = W;
  p.Hout = Hout; p.Wout = Wout;
  p.shift = (float)shift; p.C1 = (float)C1; p.C2 = (float)C2;
  for (int j = 0; j < K; ++j) {
    p.w[j] = taps[j];
    p.w2[j] = make_float2(taps[j], taps[j]);
  }
  p.dx = dx; p.dy = dy;
  p.sym = 1;
  for (int j = 0; j < K; ++j) p.sym &= (taps[j] == taps[K - 1 - j]) ? 1 : 0;
  {
    const View vx{x, N, C, H, W, p.sn, p.sc, p.sh}, vy{y, N, C, H, W, p.sn, p.sc, p.sh};
    int dx_ = 0, dy_ = 0;
    const int bw = bwd_box_width(K);
    tma = make_row_map(&p.tmx, vx, FA_F32, bw, &dx_) && make_row_map(&p.tmy, vy, FA_F32, bw, &dy_) &&
          dx_ == dy_;
    p.tma_d = tma ? dx_ : 0;
  }
  const int td = 32 * K - (K - 1);
  const SsimPlan pl = plan_rows(H, (W + td - 1) / td, p.P, device, 1, 2 * (K - 1));
  p.strips = pl.strips; p.chunks = pl.chunks; p.RH = pl.RH;
  return FA_OK;
}

int ssim_bwd_impl(const float* x, const float* y, int N, int C, int H, int W, const float* taps,
                  int K, double shift, double C1, double C2, const float* dmap,
                  const float* gscalar, const float* gs, const float* gcs, float* dx, float* dy,
                  int device, cudaStream_t st) {
  const int forms = (dmap ? 1 : 0) + (gscalar ? 1 : 0) + ((gs || gcs) ? 1 : 0);
  if (forms != 1) return FA_E_ARG;
  if ((gs != nullptr) != (gcs != nullptr)) return FA_E_ARG;
  SsimArgs p;
  bool tma = false;
  if (const int rc = bwd_setup(p, tma, x, y, N, C, H, W, taps, K, shift, C1, C2, dx, dy, device))
    return rc;
  p.dmap = dmap; p.gscalar = gscalar; p.gs = gs; p.gcs = gcs;
  const double npix = (double)p.Hout * p.Wout;
  p.grad_norm = gscalar ? (float)(1.0 / (npix * p.P)) : (gs ? (float)(1.0 / npix) : 1.0f);
  if (dmap) return bwd_g<G_MAP>(p, tma, K, device, st);
  if (gscalar) return bwd_g<G_SCALAR>(p, tma, K, device, st);
  return bwd_g<G_PLANE>(p, tma, K, device, st);
}

size_t ssim_loss_grad_ws_bytes(int N, int C, int H, int W, int K, int device) {
  const int td = 32 * K - (K - 1);
  const SsimPlan pl = plan_rows(H, (W + td - 1) / td, N * C, device, 1, 2 * (K - 1));
  return FAB_COUNTER_BYTES + sizeof(double) * (size_t)N * C * pl.strips * pl.chunks;
}

int ssim_loss_grad_impl(const float* x, const float* y, int N, int C, int H, int W,
                        const float* taps, int K, double shift, double C1, double C2,
                        double upstream, void* ws, size_t ws_bytes, double* out_plane_s,
                        double* out_per_image, double* out_total, float* dx, float* dy,
                        int device, cudaStream_t st) {
  if (!ws) return FA_E_ARG;
  SsimArgs p;
  bool tma = false;
  if (const int rc = bwd_setup(p, tma, x, y, N, C, H, W, taps, K, shift, C1, C2, dx, dy, device))
    return rc;
  const size_t nb = (size_t)p.P * p.strips * p.chunks;
  if (ws_bytes < FAB_COUNTER_BYTES + sizeof(double) * nb) return FA_E_ARG;
  p.counter = static_cast<unsigned int*>(ws);
  p.part_s = reinterpret_cast<double*>(static_cast<char*>(ws) + FAB_COUNTER_BYTES);
  p.out_plane_s = out_plane_s; p.out_per_image = out_per_image; p.out_total = out_total;
  p.grad_norm = (float)(upstream / ((double)p.Hout * p.Wout * p.P));
  return bwd_g<G_SCALAR, true>(p, tma, K, device, st);
}

}  // namespace fab
