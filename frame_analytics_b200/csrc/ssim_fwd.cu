// SSIM forward on sm_100a, host side: plans, TMA maps and dispatch.
// Replaces the reference's host path of ssim_fused_kernel
// (fa_cuda.cu:1167-1283).  Kernel: ssim_fwd.cuh.
#include "ssim_fwd.cuh"

namespace fab {

int fwd_dw_dispatch(const SsimArgs& p, int dtype, bool cs, int K, int device, cudaStream_t st);

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

static SsimPlan fwd_plan(int Hout, int Wout, int K, int planes, int device) {
  const int nt = 32 * K;
  return plan_rows(Hout, (Wout + nt - 1) / nt, planes, device, 2, K - 1);
}

size_t ssim_ws_bytes(int planes, int Hout, int Wout, int K, int device) {
  const SsimPlan pl = fwd_plan(Hout, Wout, K, planes, device);
  // partial sums: SSIM, cs, squared differences and the GMSD pair (8 bytes each per block)
  return FAB_COUNTER_BYTES + 5 * sizeof(double) * (size_t)planes * pl.strips * pl.chunks;
}

template <typename T, bool CS, int STAGE>
static int fwd_k(const SsimArgs& p, int K, int device, cudaStream_t st) {
  switch (K) {
    case 11: return launch_fwd<T, 11, CS, STAGE>(p, device, st);
    case 9: return launch_fwd<T, 9, CS, STAGE>(p, device, st);
    case 7: return launch_fwd<T, 7, CS, STAGE>(p, device, st);
    case 5: return launch_fwd<T, 5, CS, STAGE>(p, device, st);
    case 3: return launch_fwd<T, 3, CS, STAGE>(p, device, st);
    default: return FA_E_WINDOW;
  }
}

template <typename T, int STAGE>
static int fwd_sq_k(const SsimArgs& p, int K, int device, cudaStream_t st) {
  switch (K) {
    case 11: return launch_fwd<T, 11, false, STAGE, true>(p, device, st);
    case 9: return launch_fwd<T, 9, false, STAGE, true>(p, device, st);
    case 7: return launch_fwd<T, 7, false, STAGE, true>(p, device, st);
    case 5: return launch_fwd<T, 5, false, STAGE, true>(p, device, st);
    case 3: return launch_fwd<T, 3, false, STAGE, true>(p, device, st);
    default: return FA_E_WINDOW;
  }
}

template <typename T>
static int fwd_dispatch(const SsimArgs& p, int stage, bool cs, int K, int device,
                        cudaStream_t st) {
  if (p.part_sq) {
    if (stage == STAGE_TMA) return fwd_sq_k<T, STAGE_TMA>(p, K, device, st);
    if (stage == STAGE_GENERIC) return fwd_sq_k<T, STAGE_GENERIC>(p, K, device, st);
    return FA_E_ARG;  // luma: the squared differences are of the RGB planes
  }
  if (stage == STAGE_TMA)
    return cs ? fwd_k<T, true, STAGE_TMA>(p, K, device, st)
              : fwd_k<T, false, STAGE_TMA>(p, K, device, st);
  if (stage == STAGE_LUMA)
    return cs ? fwd_k<T, true, STAGE_LUMA>(p, K, device, st)
              : fwd_k<T, false, STAGE_LUMA>(p, K, device, st);
  return cs ? fwd_k<T, true, STAGE_GENERIC>(p, K, device, st)
            : fwd_k<T, false, STAGE_GENERIC>(p, K, device, st);
}

// ---------------------------------------------------------------------------
// TMA maps
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
  }
  return fn;
}

bool make_row_map(CUtensorMap* map, const View& v, int dtype, int box_w, int* d) {
  static const int esz[6] = {1, 2, 2, 4, 8, 2};
  static const CUtensorMapDataType dts[6] = {
      CU_TENSOR_MAP_DATA_TYPE_UINT8, CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
      CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
      CU_TENSOR_MAP_DATA_TYPE_FLOAT64,
      CU_TENSOR_MAP_DATA_TYPE_UINT16};
  if (dtype < 0 || dtype > 5) return false;
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const long long E = esz[dtype];
  const uintptr_t a = reinterpret_cast<uintptr_t>(v.data);
  const uintptr_t b = a & ~(uintptr_t)15;
  if ((a - b) % E) return false;
  *d = (int)((a - b) / E);
  // strides of singleton dimensions are never used: give them a legal value
  long long sh = v.sh * E, sc = v.sc * E, sn = v.sn * E;
  if (v.c == 1) sc = ((sh * v.h + 15) / 16) * 16;
  if (v.n == 1) sn = ((sc * v.c + 15) / 16) * 16;
  const long long lim = 1LL << 40;
  if (sh % 16 || sc % 16 || sn % 16 || sh <= 0 || sc <= 0 || sn <= 0 || sh >= lim ||
      sc >= lim || sn >= lim)
    return false;
  if ((box_w * E) % 16 || box_w > 256) return false;
  const cuuint64_t dims[4] = {(cuuint64_t)(v.w + *d), (cuuint64_t)v.h, (cuuint64_t)v.c,
                              (cuuint64_t)v.n};
  const cuuint64_t strides[3] = {(cuuint64_t)sh, (cuuint64_t)sc, (cuuint64_t)sn};
  const cuuint32_t box[4] = {(cuuint32_t)box_w, 1, 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(map, dts[dtype], 4, reinterpret_cast<void*>(b), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_map_3d_u64(CUtensorMap* map, const void* base, unsigned long long d0,
                     unsigned long long d1, unsigned long long d2, unsigned long long s1,
                     unsigned long long s2, int b0, int b1) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || reinterpret_cast<uintptr_t>(base) % 16 || s1 % 16 || s2 % 16) return false;
  if (b0 <= 0 || b0 > 256 || b1 <= 0 || b1 > 256 || (b0 * 8) % 16) return false;
  const cuuint64_t dims[3] = {d0, d1, d2};
  const cuuint64_t strides[2] = {s1, s2};
  const cuuint32_t box[3] = {(cuuint32_t)b0, (cuuint32_t)b1, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

template <int KW>
static int box_width(int dtype) {
  switch (dtype) {
    case FA_U8: return Raw<unsigned char, KW>::BW;
    case FA_F16: return Raw<f16_t, KW>::BW;
    case FA_BF16: return Raw<bf16_t, KW>::BW;
    case FA_F32: return Raw<float, KW>::BW;
    case FA_U16: return Raw<unsigned short, KW>::BW;
    default: return Raw<double, KW>::BW;
  }
}

static int box_width_k(int K, int dtype) {
  switch (K) {
    case 11: return box_width<11>(dtype);
    case 9: return box_width<9>(dtype);
    case 7: return box_width<7>(dtype);
    case 5: return box_width<5>(dtype);
    default: return box_width<3>(dtype);
  }
}

int ssim_fwd_impl(const View& x, const View& y, int dtype, const double* luma, const float* taps,
                  int K, double shift, double C1, double C2, float* map_out, void* ws,
                  size_t ws_bytes, double* out_plane_s, double* out_plane_cs,
                  double* out_per_image, double* out_total, int device, cudaStream_t st,
                  const SqOut* sq, const float* wdev, const GmOut* gm) {
  if (!x.data || !y.data || (!taps && !wdev) || !ws) return FA_E_ARG;
  if (gm && (wdev || luma || out_plane_cs || map_out)) return FA_E_ARG;
  if (wdev && (sq || luma)) return FA_E_ARG;
  if (sq && (luma || out_plane_cs)) return FA_E_ARG;
  if (x.n <= 0 || x.c <= 0 || x.h <= 0 || x.w <= 0) return FA_E_SHAPE;
  if (x.n != y.n || x.c != y.c || x.h != y.h || x.w != y.w) return FA_E_SHAPE;
  if (x.sn != y.sn || x.sc != y.sc || x.sh != y.sh) return FA_E_SHAPE;
  if (K < 3 || K > FA_MAX_WIN || (K & 1) == 0) return FA_E_WINDOW;
  if (luma && x.c != 3) return FA_E_SHAPE;
  const int Hout = x.h - K + 1, Wout = x.w - K + 1;
  if (Hout <= 0 || Wout <= 0) return FA_E_SHAPE;
  SsimArgs p{};
  p.err = wait_error_word();
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
  if (taps) {
    for (int j = 0; j < K; ++j) {
      p.w[j] = taps[j];
      p.w2[j] = make_float2(taps[j], taps[j]);
    }
  }
  p.wdev = wdev;
  const SsimPlan pl = fwd_plan(Hout, Wout, K, p.P, device);
  p.strips = pl.strips; p.chunks = pl.chunks; p.RH = pl.RH;
  const size_t nb = (size_t)p.P * pl.strips * pl.chunks;
  if (ws_bytes < FAB_COUNTER_BYTES + (gm ? 5 : (sq ? 3 : 2)) * sizeof(double) * nb)
    return FA_E_ARG;
  p.counter = static_cast<unsigned int*>(ws);
  p.part_s = reinterpret_cast<double*>(static_cast<char*>(ws) + FAB_COUNTER_BYTES);
  p.part_cs = out_plane_cs ? p.part_s + nb : nullptr;
  if (sq) {
    p.part_sq = p.part_s + 2 * nb;
    p.psnr_bias = sq->psnr_bias;
    p.out_mse_per_image = sq->mse_per_image;
    p.out_mse_total = sq->mse_total;
    p.out_psnr_per_image = sq->psnr_per_image;
    p.out_psnr_total = sq->psnr_total;
    p.out_ssd_per_image = (dtype == FA_U8 || dtype == FA_U16) ? sq->ssd_per_image : nullptr;
  }
  if (gm) {
    p.part_g = p.part_s + 3 * nb;
    p.gT = (float)gm->T;
    p.geps = (float)gm->eps;
    p.gHo = x.h / 2 - 2;
    p.gWo = x.w / 2 - 2;
    p.out_gms_per_image = gm->gms_per_image;
    p.out_gmsd_per_image = gm->gmsd_per_image;
    if (p.gHo <= 0 || p.gWo <= 0 || K != 11 || p.gWo > pl.strips * (Geo<11>::NT / 2))
      return FA_E_SHAPE;
  }
  p.map_out = map_out;
  p.out_plane_s = out_plane_s; p.out_plane_cs = out_plane_cs;
  p.out_per_image = out_per_image; p.out_total = out_total;
  const bool cs = out_plane_cs != nullptr;
  if (dtype < 0 || dtype > 5) return FA_E_DTYPE;
  int stage = luma ? STAGE_LUMA : STAGE_GENERIC;
  if (wdev) return fwd_dw_dispatch(p, dtype, cs, K, device, st);
  bool sym = true;  // the TMA kernels read only the first (K+1)/2 taps
  for (int j = 0; j < K; ++j) sym = sym && taps[j] == taps[K - 1 - j];
  if (!luma && sym) {
    const int bw = box_width_k(K, dtype);
    int dx = 0, dy = 0;
    if (make_row_map(&p.tmx, x, dtype, bw, &dx) && make_row_map(&p.tmy, y, dtype, bw, &dy) &&
        dx == dy) {
      stage = STAGE_TMA;
      p.tma_d = dx;
    }
  }
  if (gm) {
    if (stage != STAGE_TMA) return FA_E_SHAPE;
    if (dtype == FA_U8)
      return sq ? launch_fwd<unsigned char, 11, false, STAGE_TMA, true, false, true>(p, device, st)
                : launch_fwd<unsigned char, 11, false, STAGE_TMA, false, false, true>(p, device, st);
    if (dtype == FA_F32)
      return sq ? launch_fwd<float, 11, false, STAGE_TMA, true, false, true>(p, device, st)
                : launch_fwd<float, 11, false, STAGE_TMA, false, false, true>(p, device, st);
    return FA_E_DTYPE;
  }
  switch (dtype) {
    case FA_U8: return fwd_dispatch<unsigned char>(p, stage, cs, K, device, st);
    case FA_F16: return fwd_dispatch<f16_t>(p, stage, cs, K, device, st);
    case FA_BF16: return fwd_dispatch<bf16_t>(p, stage, cs, K, device, st);
    case FA_F32: return fwd_dispatch<float>(p, stage, cs, K, device, st);
    case FA_U16: return fwd_dispatch<unsigned short>(p, stage, cs, K, device, st);
    default: return fwd_dispatch<double>(p, stage, cs, K, device, st);
  }
}

// Whether ssim_fwd_impl can add GMSD (2x2 pool) to this pair's SSIM pass: an
// 11-tap symmetric window, uint8 or float32 rows a TMA map can describe, and
// a GMS map no wider than the strips' owned columns.
bool ssim_gmsd_fusable(const View& x, const View& y, int dtype, int K, int device) {
  if (K != 11 || (dtype != FA_U8 && dtype != FA_F32)) return false;
  if (x.h < 11 || x.w < 11 || x.h / 2 - 2 <= 0 || x.w / 2 - 2 <= 0) return false;
  if (x.sn != y.sn || x.sc != y.sc || x.sh != y.sh) return false;
  const SsimPlan pl = fwd_plan(x.h - 10, x.w - 10, 11, x.n * x.c, device);
  if (x.w / 2 - 2 > pl.strips * (Geo<11>::NT / 2)) return false;
  CUtensorMap mx, my;
  const int bw = box_width_k(11, dtype);
  int dx = 0, dy = 0;
  return make_row_map(&mx, x, dtype, bw, &dx) && make_row_map(&my, y, dtype, bw, &dy) && dx == dy;
}

}  // namespace fab
