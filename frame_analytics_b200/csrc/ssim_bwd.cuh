// Fused SSIM backward on sm_100a: one launch, no frame-sized scratch.
// This header holds the general kernel (any window, register or TMA
// staging); the warp-specialised kernel and the host side are ssim_bwd.cu.
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
#pragma once

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
__device__ __forceinline__ void ssim_bwd_body(const SsimArgs& p) {
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
      mbar_wait(&s_bar[0], m & 1, p.err);
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
    if constexpr (TMA) mbar_wait(&s_bar[1], m & 1, p.err);
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

// DW: taps from `wdev` (register staging only; see load_device_taps).
template <int KW, bool DX, bool DY, int GMODE, int STAGE, bool FWD, bool DW = false>
__global__ void __launch_bounds__(32 * KW, 1) ssim_bwd_kernel(const __grid_constant__ SsimArgs p) {
  if constexpr (DW) {
    static_assert(STAGE == STAGE_GENERIC, "device taps use register staging");
    SsimArgs q = p;
    load_device_taps<KW>(q);
    ssim_bwd_body<KW, DX, DY, GMODE, STAGE, FWD>(q);
  } else {
    ssim_bwd_body<KW, DX, DY, GMODE, STAGE, FWD>(p);
  }
}

template <int KW, bool DX, bool DY, int GMODE, int STAGE, bool FWD, bool DW = false>
static int launch_bwd_general(const SsimArgs& p, int device, cudaStream_t st) {
  dim3 grid(p.strips, p.chunks, p.P);
  auto kern = ssim_bwd_kernel<KW, DX, DY, GMODE, STAGE, FWD, DW>;
  const size_t sm = BwdGeo<KW>::kBytes;
  static bool done[64] = {false};
  FAB_TRY(ensure_smem(kern, sm, device, done));
  kern<<<grid, 32 * KW, sm, st>>>(p);
  FAB_LAUNCH_CHECK();
  return FA_OK;
}

}  // namespace fab
