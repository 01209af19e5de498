// Fused SSIM backward on sm_100a: the warp-specialised kernel and the host
// side (the general kernel and the math: ssim_bwd.cuh).
#include "ssim_bwd.cuh"

namespace fab {

int bwd_dw_dispatch(const SsimArgs& p, int gmode, int K, int device, cudaStream_t st);

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
        mbar_wait(&s_bar, m & 1, p.err);
        hblur_raw<KW>(p, sX + warp * R::RP + sofs + lane * KW, sY + warp * R::RP + sofs + lane * KW,
                      sH + warp * NT + lane * KW);
      }
      __syncthreads();
      if (m < iters) {
        if (m + 1 < iters) stage_tma<float, KW>(p, pn, pc, i0 + (m + 1) * KW, xs0, sX, sY, &s_bar);
        const int o0 = i0 + m * KW - (KW - 1);  // moment row of slot 0
        float fs = 0.f;
        // CHK: per-row tests; interior batches (every row a valid, owned
        // moment row) skip them.  FLAT (interior, no per-position upstream
        // gradient to load): no branches at all; a column outside the moment
        // strip gets zero coefficients and adds nothing, by select.
        auto rows_step = [&](auto chk, auto flat) {
          constexpr bool CHK = decltype(chk)::value;
          constexpr bool FLAT = decltype(flat)::value;
#pragma unroll
          for (int k = 0; k < KW; ++k) {
            ring[k] = sH[k * NT + t];
            const int o = o0 + k;
            float4 cf = make_float4(0.f, 0.f, 0.f, 0.f);
            if (FLAT || (q_ok && (!CHK || (m * KW + k >= KW - 1 && o >= 0 && o < p.Hout)))) {
              const Moments mo = moments(p, vblur_at<KW, 4, true>(p, ring, k));
              // one approximate reciprocal (a few ulp) serves S, cs and the
              // coefficients
              const float inv = __fdividef(1.0f, mo.B1 * mo.B2);
              const float iB1 = mo.B2 * inv;
              const float iB2 = mo.B1 * inv;
              const float S = mo.A1 * mo.A2 * inv;
              const float kk = 2.f * mo.A2 * inv;
              if (FLAT) {
                if (FWD) fs += own_col ? S : 0.f;
              } else if (FWD && own_col && (!CHK || (o >= r0 && o < r0 + rows))) {
                fs += S;
              }
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
              if (FLAT && !q_ok) cf = make_float4(0.f, 0.f, 0.f, 0.f);
            }
            sC[k * B::SCW + t] = cf;
          }
        };
        const bool interior = m >= 1 && o0 >= 0 && o0 + KW - 1 < p.Hout &&
                              (!FWD || (o0 >= r0 && o0 + KW - 1 < r0 + rows));
        if (interior && GMODE != G_MAP) rows_step(std::false_type{}, std::true_type{});
        else if (interior) rows_step(std::false_type{}, std::false_type{});
        else rows_step(std::true_type{}, std::false_type{});
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
    FAB_LAUNCH_CHECK();
    return FA_OK;
  }
  return launch_bwd_general<KW, DX, DY, GMODE, STAGE, FWD>(p, device, st);
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
                     float* dx, float* dy, int device, const float* wdev = nullptr) {
  if (!x || !y || (!taps && !wdev)) return FA_E_ARG;
  if (!dx && !dy) return FA_E_ARG;
  if (N <= 0 || C <= 0 || H <= 0 || W <= 0) return FA_E_SHAPE;
  if (K < 3 || K > FA_MAX_WIN || (K & 1) == 0) return FA_E_WINDOW;
  const int Hout = H - K + 1, Wout = W - K + 1;
  if (Hout <= 0 || Wout <= 0) return FA_E_SHAPE;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 3u) return FA_E_ARG;
  p = SsimArgs{};
  p.err = wait_error_word();
  p.x = reinterpret_cast<const char*>(x);
  p.y = reinterpret_cast<const char*>(y);
  p.N = N; p.C = C; p.H = H; p.W = W;
  p.Cm = C; p.P = N * C;
  if (p.P > 65535) return FA_E_SHAPE;
  p.sn = (long long)C * H * W; p.sc = (long long)H * W; p.sh = W;
  p.Hout = Hout; p.Wout = Wout;
  p.shift = (float)shift; p.C1 = (float)C1; p.C2 = (float)C2;
  p.dx = dx; p.dy = dy;
  p.wdev = wdev;
  if (taps) {
    for (int j = 0; j < K; ++j) {
      p.w[j] = taps[j];
      p.w2[j] = make_float2(taps[j], taps[j]);
    }
    p.sym = 1;
    for (int j = 0; j < K; ++j) p.sym &= (taps[j] == taps[K - 1 - j]) ? 1 : 0;
  }
  if (wdev) {
    tma = false;  // device taps: register staging, general kernel
  } else {
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
                  int device, cudaStream_t st, const float* wdev) {
  const int forms = (dmap ? 1 : 0) + (gscalar ? 1 : 0) + ((gs || gcs) ? 1 : 0);
  if (forms != 1) return FA_E_ARG;
  if ((gs != nullptr) != (gcs != nullptr)) return FA_E_ARG;
  SsimArgs p;
  bool tma = false;
  if (const int rc =
          bwd_setup(p, tma, x, y, N, C, H, W, taps, K, shift, C1, C2, dx, dy, device, wdev))
    return rc;
  p.dmap = dmap; p.gscalar = gscalar; p.gs = gs; p.gcs = gcs;
  const double npix = (double)p.Hout * p.Wout;
  p.grad_norm = gscalar ? (float)(1.0 / (npix * p.P)) : (gs ? (float)(1.0 / npix) : 1.0f);
  if (wdev) return bwd_dw_dispatch(p, dmap ? G_MAP : (gscalar ? G_SCALAR : G_PLANE), K, device, st);
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
