/*
 * frame_analytics_b200 -- C ABI of the B200 (sm_100a) full-reference metric kernels.
 *
 * Two blocks of entry points live in libfa_b200.so:
 *
 *  1. `fa_cuda_*`: drop-in replacements for every CUDA entry point the
 *     reference binds through ctypes (frame_analytics/csrc/fa_abi.h:118-200,
 *     prototypes in frame_analytics/_cabi.py:414-462).  Same names, same
 *     argument meaning, same status codes, so the reference's own loader can
 *     bind this library in place of its libfa_cuda.  Scratch arguments the
 *     reference needs (`partial`, `aux`) are accepted; `aux` is unused because
 *     the backward here recomputes the moments instead of staging them.
 *
 *  2. `fa_b200_*`: the extended boundary the Python layer in this package
 *     uses.  Inputs are strided views (crop_border needs no copy), luma is
 *     folded into the loads, finalisation happens inside the reduction launch,
 *     integer sums come back as exact uint64, and the backward has no
 *     frame-sized temporaries.
 *
 * Conventions (kept from the reference, fa_abi.h:12-21):
 *   - every entry point returns an int: 0 = ok, 1..7 = library codes below,
 *     negative = -(cudaError_t);
 *   - the caller owns every buffer, scratch included; nothing here calls
 *     cudaMalloc/cudaFree and nothing synchronises the host;
 *   - `device` is an explicit ordinal (set and restored around the launch),
 *     `stream` is a cudaStream_t passed as void*;
 *   - launches are asynchronous on `stream`.
 *
 * Scratch ("workspace") of the fa_b200_* calls: a byte buffer whose size the
 * matching *_workspace_bytes query returns.  Its first 256 bytes hold the
 * grid-completion counters the single-launch finalisers use; they must be
 * zero when the call starts, and every call leaves them zero again, so a
 * workspace zeroed once can be reused by any number of calls issued in order
 * on one stream.  Two calls that may run concurrently need two workspaces.
 */
#ifndef FA_B200_H
#define FA_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(_WIN32)
#define FA_B200_API __declspec(dllexport)
#else
#define FA_B200_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Same value as the reference's FA_ABI_VERSION (fa_abi.h:41): the fa_cuda_*
 * block below keeps that ABI. */
#define FA_ABI_VERSION 1
/* Version of the fa_b200_* block. */
#define FA_B200_ABI_VERSION 1

/* dtype codes (fa_abi.h:43-48) */
#define FA_U8 0
#define FA_F16 1
#define FA_BF16 2
#define FA_F32 3
#define FA_F64 4
/* Extension, no counterpart in the reference (which widens uint16 to float32
 * in torch first): uint16 samples, e.g. 10-16-bit video.  Accepted by the
 * fa_b200_* calls; MSE / L1 of uint16 are exact integer sums, like uint8. */
#define FA_U16 5

/* pixel-loss selector (fa_abi.h:50-54) */
#define FA_OP_MSE 0
#define FA_OP_L1 1
#define FA_OP_CHARB 2 /* param = eps^2 */
#define FA_OP_HUBER 3 /* param = delta */

/* status codes (fa_abi.h:56-64); negative returns are -(cudaError_t) */
#define FA_OK 0
#define FA_E_DTYPE 1
#define FA_E_SHAPE 2
#define FA_E_WINDOW 3
#define FA_E_OP 4
#define FA_E_ARG 5
#define FA_E_INTERNAL 6
#define FA_E_NOCUDA 7
/* Extension, no counterpart in the reference: a bounded device-side wait (a
 * TMA row copy that never completed) gave up.  Kernels run asynchronously, so
 * the code is returned by the first compute call made after the failing
 * kernel has finished; that call enqueues nothing.  The failing kernel's
 * outputs are garbage. */
#define FA_E_TIMEOUT 8

/* "not an MSE reduction, skip the dB conversion" (fa_abi.h:67) */
#define FA_PSNR_NONE (-1.0e300)

/* largest Gaussian window; odd widths 3..11 are instantiated (fa_abi.h:71) */
#define FA_MAX_WIN 11

/* ======================================================================= */
/* 1. reference-compatible block                                            */
/* ======================================================================= */

/* replaces fa_cuda_abi_version, fa_abi.h:118 */
FA_B200_API int fa_cuda_abi_version(void);
/* replaces fa_cuda_error_string, fa_abi.h:119 */
FA_B200_API const char* fa_cuda_error_string(int code);
/* replaces fa_cuda_device_count, fa_abi.h:120 */
FA_B200_API int fa_cuda_device_count(int* out_count);

/* replaces fa_cuda_pixel_workspace, fa_abi.h:122-123.
 * out_bpi: columns of the [n_images, bpi] float64 `partial` scratch. */
FA_B200_API int fa_cuda_pixel_workspace(int64_t n_images, int64_t n_per_image,
                                        int device, int* out_bpi);

/* replaces fa_cuda_pixel_reduce, fa_abi.h:127-134.  Contiguous images. */
FA_B200_API int fa_cuda_pixel_reduce(const void* a, const void* b, int dtype,
                                     int64_t n_images, int64_t n_per_image,
                                     int op, double param, double psnr_bias,
                                     double* partial, int bpi,
                                     double* out_per_image, double* out_total,
                                     double* out_psnr_per_image,
                                     double* out_psnr_total, int device,
                                     void* stream);

/* replaces fa_cuda_ssim_workspace, fa_abi.h:136 */
FA_B200_API int fa_cuda_ssim_workspace(int H, int W, int K, int* out_bpp);

/* replaces fa_cuda_ssim, fa_abi.h:139-146.  partial: [N*C, bpp] float64.
 * `win` is the device window, as in the reference; the SSIM entry points of
 * this block copy it to the host once per (device, pointer, K) and cache it,
 * so the first call with a given window synchronises (make it outside any
 * stream capture). */
FA_B200_API int fa_cuda_ssim(const void* x, const void* y, int dtype, int N,
                             int C, int H, int W, const float* win, int K,
                             double shift, double C1, double C2,
                             float* map_out, double* partial, int bpp,
                             double* out_per_image, double* out_total,
                             int device, void* stream);

/* replaces fa_cuda_ssim_cs, fa_abi.h:149-155.  out_s/out_cs: N*C plane means. */
FA_B200_API int fa_cuda_ssim_cs(const void* x, const void* y, int dtype, int N,
                                int C, int H, int W, const float* win, int K,
                                double shift, double C1, double C2,
                                double* partial, double* partial_cs, int bpp,
                                double* out_s, double* out_cs, int device,
                                void* stream);

/* replaces fa_cuda_ssim_backward, fa_abi.h:161-168.  `aux` is accepted and
 * ignored (may be null): the fused backward keeps no frame-sized scratch. */
FA_B200_API int fa_cuda_ssim_backward(const float* x, const float* y,
                                      const float* dL_dmap,
                                      const float* grad_scalar,
                                      const float* win, int K, int N, int C,
                                      int H, int W, double shift, double C1,
                                      double C2, float* aux, float* dx,
                                      float* dy, int device, void* stream);

/* replaces fa_cuda_ssim_cs_backward, fa_abi.h:171-177.  `aux` ignored. */
FA_B200_API int fa_cuda_ssim_cs_backward(const float* x, const float* y,
                                         const float* gs, const float* gcs,
                                         const float* win, int K, int N,
                                         int C, int H, int W, double shift,
                                         double C1, double C2, float* aux,
                                         float* dx, float* dy, int device,
                                         void* stream);

/* replaces fa_cuda_gmsd_workspace, fa_abi.h:179 */
FA_B200_API int fa_cuda_gmsd_workspace(int H, int W, int downsample,
                                       int* out_bpp);

/* replaces fa_cuda_gmsd, fa_abi.h:182-187 */
FA_B200_API int fa_cuda_gmsd(const void* x, const void* y, int dtype, int N,
                             int C, int H, int W, double Tc, double eps,
                             int downsample, double* psum, double* psumsq,
                             int bpp, double* out_mean, double* out_std,
                             int device, void* stream);

/* ======================================================================= */
/* 2. extended block                                                        */
/* ======================================================================= */

/* A batch of images as a strided 4-D view (N, C, H, W).  Strides are in
 * elements; the W stride is 1.  `data` points at element (0,0,0,0). */
typedef struct fa_view {
  const void* data;
  int32_t dtype;
  int32_t n, c, h, w;
  int32_t pad_;
  int64_t stride_n, stride_c, stride_h;
} fa_view;

/* Luma projection folded into the loads: Y = k[0]*R + k[1]*G + k[2]*B + k[3]
 * (k[3] is the offset already multiplied by the data range).  Pass NULL for
 * "no luma"; with luma the view must have c == 3 and the metric sees one
 * channel.  Mirrors functional.rgb_to_luma (functional.py:213-237). */

FA_B200_API int fa_b200_abi_version(void);

/* Bytes of workspace fa_b200_pixel_reduce needs for `n_images` images. */
FA_B200_API int fa_b200_pixel_workspace_bytes(int n_images, int device,
                                              size_t* out_bytes);

/* One-launch pixel reduction (MSE / L1 / Charbonnier / Huber), PSNR on top.
 * Replaces the pair fa_cuda_pixel_reduce + finalize (fa_cuda.cu:1078-1156)
 * and the torch luma materialisation (functional.py:267-271).
 *   out_per_image[n], out_total[0]       : means (nullable)
 *   out_psnr_per_image[n], out_psnr_total: dB, when psnr_bias != FA_PSNR_NONE
 *   out_isum_per_image[n]                : exact integer sums (uint8 MSE/L1
 *                                          without luma only; else ignored) */
FA_B200_API int fa_b200_pixel_reduce(const fa_view* a, const fa_view* b,
                                     const double* luma, int op, double param,
                                     double psnr_bias, void* workspace,
                                     size_t workspace_bytes,
                                     double* out_per_image, double* out_total,
                                     double* out_psnr_per_image,
                                     double* out_psnr_total,
                                     uint64_t* out_isum_per_image, int device,
                                     void* stream);

/* Bytes of workspace fa_b200_ssim needs. */
FA_B200_API int fa_b200_ssim_workspace_bytes(int n, int c, int h, int w, int K,
                                             int device, size_t* out_bytes);

/* Fused SSIM forward in one launch.  Replaces fa_cuda_ssim / fa_cuda_ssim_cs
 * + finalize (fa_cuda.cu:1167-1283).  All outputs nullable:
 *   map_out          [N, C', Hout, Wout] float32 SSIM map
 *   out_plane_s/cs   [N*C'] per-plane means of SSIM and of its cs factor
 *   out_per_image    [N] mean over C' planes; out_total: batch mean
 * (C' = 1 with luma, else C).
 * taps_host: the K float32 taps of the 1-D window, in HOST memory, read
 * during the call (they travel in the kernel parameters). */
FA_B200_API int fa_b200_ssim(const fa_view* x, const fa_view* y,
                             const double* luma, const float* taps_host, int K,
                             double shift, double C1, double C2,
                             float* map_out, void* workspace,
                             size_t workspace_bytes, double* out_plane_s,
                             double* out_plane_cs, double* out_per_image,
                             double* out_total, int device, void* stream);

/* SSIM, MSE and PSNR from one read of the frame pair (the reference's
 * StreamingMetrics default set, modules.py:373-402, which runs mse and ssim
 * as separate kernels, fa_cuda.cu:1078-1156 and 1167-1283).  SSIM outputs as
 * fa_b200_ssim (no map, no cs, no luma); the squared differences are summed
 * over every input sample while the SSIM kernel stages it: exact uint64 sums
 * for uint8 (out_ssd_per_image, [N]; NULL for other dtypes), float terms
 * summed in double otherwise (double terms for f64), as
 * fa_b200_pixel_reduce with FA_OP_MSE.  MSE per image / batch and PSNR
 * (psnr_bias - 10 log10 mse) as there.  Every output is nullable.  The
 * workspace is sized by fa_b200_ssim_workspace_bytes. */
FA_B200_API int fa_b200_ssim_mse(const fa_view* x, const fa_view* y,
                                 const float* taps_host, int K, double shift,
                                 double C1, double C2, double psnr_bias,
                                 void* workspace, size_t workspace_bytes,
                                 double* out_plane_s, double* out_per_image,
                                 double* out_total, double* out_mse_per_image,
                                 double* out_mse_total,
                                 double* out_psnr_per_image,
                                 double* out_psnr_total,
                                 uint64_t* out_ssd_per_image, int device,
                                 void* stream);

/* No single counterpart in the reference: the SSIM and GMSD of config 4
 * (and optionally MSE / PSNR) from ONE read of the frame pair.  The
 * reference's StreamingMetrics scores them with separate kernels
 * (modules.py:373-402; SSIM fa_cuda.cu:1167-1223, GMSD fa_cuda.cu:1426-1466),
 * reading every frame twice.  Here the SSIM kernel's staged rows also feed a
 * 2x2-pooled Prewitt pass.  GMSD semantics are fa_b200_gmsd's with
 * downsample=1: q over the (H/2-2) x (W/2-2) map of every plane, pooled over
 * the image's planes; out_gms_per_image = mean q, out_gmsd_per_image = its
 * population std.  SSIM and MSE / PSNR outputs as fa_b200_ssim_mse; the
 * MSE / PSNR pass runs only when one of its outputs is non-NULL.  Every
 * output is nullable.  Serves the pairs fa_b200_ssim_gmsd_fusable accepts
 * (11-tap symmetric window, uint8 or float32, rows a TMA map can describe);
 * others return FA_E_SHAPE.  Workspace: fa_b200_ssim_workspace_bytes. */
FA_B200_API int fa_b200_ssim_gmsd_fusable(const fa_view* x, const fa_view* y, int K,
                                          int device, int* out_ok);
FA_B200_API int fa_b200_ssim_gmsd(const fa_view* x, const fa_view* y,
                                  const float* taps_host, int K, double shift,
                                  double C1, double C2, double gmsd_T,
                                  double gmsd_eps, double psnr_bias,
                                  void* workspace, size_t workspace_bytes,
                                  double* out_plane_s, double* out_per_image,
                                  double* out_total, double* out_gms_per_image,
                                  double* out_gmsd_per_image,
                                  double* out_mse_per_image, double* out_mse_total,
                                  double* out_psnr_per_image,
                                  double* out_psnr_total,
                                  uint64_t* out_ssd_per_image, int device,
                                  void* stream);

/* SSIM loss value and gradient in one pass (training steps).  No single
 * counterpart in the reference: it runs its forward (fa_cuda_ssim,
 * fa_cuda.cu:1167-1283) and later its backward (fa_cuda_ssim_backward,
 * fa_cuda.cu:1299-1414), both reading x and y and recomputing the moments.
 * Since d(mean SSIM)/dx is linear in the upstream scalar, this call returns
 * the SSIM means (as fa_b200_ssim: out_plane_s [N*C], out_per_image [N],
 * out_total [1], each nullable) together with dx / dy = the gradient of the
 * batch-mean SSIM (out_total) for the upstream gradient `upstream` (1 for
 * the unit gradient; -1 gives the gradient of a loss 1 - SSIM directly); the
 * caller rescales by its real upstream gradient (fa_b200_grad_scale).  Per
 * image n,
 * d(out_per_image[n])/dx = N * dx restricted to image n.
 * x, y: float32 contiguous [N, C, H, W]; dx / dy nullable (not both);
 * taps_host: host memory.  workspace: device memory of the size
 * fa_b200_ssim_loss_grad_workspace_bytes reports, zeroed once before first
 * use and reused only by calls serialised on one stream. */
FA_B200_API int fa_b200_ssim_loss_grad_workspace_bytes(int n, int c, int h,
                                                       int w, int K,
                                                       int device,
                                                       size_t* out_bytes);
FA_B200_API int fa_b200_ssim_loss_grad(const float* x, const float* y, int N,
                                       int C, int H, int W,
                                       const float* taps_host, int K,
                                       double shift, double C1, double C2,
                                       double upstream, void* workspace,
                                       size_t workspace_bytes,
                                       double* out_plane_s,
                                       double* out_per_image,
                                       double* out_total, float* dx,
                                       float* dy, int device, void* stream);

/* out = in * (s * mult), elementwise over n images of per_image floats: s is
 * one device double (per_image_scale = 0) or n of them (one per image).
 * Applies the upstream gradient to the unit gradient fa_b200_ssim_loss_grad
 * returns (mult = N for per-image upstream gradients).  No counterpart in
 * the reference, whose backward receives the upstream gradient directly.
 * in and out may alias; in place, samples whose factor is exactly 1 are
 * left untouched (a single scale of 1 returns at once). */
FA_B200_API int fa_b200_grad_scale(const float* in, long long per_image, int n,
                                   const double* s, int per_image_scale,
                                   double mult, float* out, int device,
                                   void* stream);

/* Fused SSIM backward, one launch, no scratch.  Replaces fa_cuda_ssim_backward
 * and fa_cuda_ssim_cs_backward (fa_cuda.cu:1299-1414, backend.py:429-455).
 * Upstream gradient, exactly one form:
 *   dL_dmap   [N, C, Hout, Wout]  : per map position
 *   g_scalar  [1] (device)        : d loss / d (batch-mean SSIM); scaled by
 *                                   1/(N*C*Hout*Wout) inside
 *   gs, gcs   [N*C] (device)      : d loss / d (plane-mean SSIM) and
 *                                   d loss / d (plane-mean cs) (MS-SSIM)
 * x, y: float32 contiguous [N, C, H, W].  dx / dy nullable (not both).
 * taps_host: as for fa_b200_ssim (host memory). */
FA_B200_API int fa_b200_ssim_backward(const float* x, const float* y, int N,
                                      int C, int H, int W, const float* taps_host,
                                      int K, double shift, double C1,
                                      double C2, const float* dL_dmap,
                                      const float* g_scalar, const float* gs,
                                      const float* gcs, float* dx, float* dy,
                                      int device, void* stream);

/* Bytes of workspace fa_b200_gmsd needs. */
FA_B200_API int fa_b200_gmsd_workspace_bytes(int n, int c, int h, int w,
                                             int downsample, int device,
                                             size_t* out_bytes);

/* Fused GMSD in one launch: optional 2x2 mean pool, Prewitt/3, GMS map, per
 * image mean and population std pooled over all channels.  Replaces
 * fa_cuda_gmsd + gmsd_finalize (fa_cuda.cu:926-1026, 1426-1466) and, with
 * map_out, the portable GMS map of functional._gms_map (functional.py:925-947).
 *   map_out [N, C', Hout, Wout] float32 (nullable); out_mean (GMS) / out_std
 *   (GMSD): [N] float64. */
FA_B200_API int fa_b200_gmsd(const fa_view* x, const fa_view* y,
                             const double* luma, double T, double eps,
                             int downsample, void* workspace,
                             size_t workspace_bytes, float* map_out,
                             double* out_mean, double* out_std, int device,
                             void* stream);

/* Gradient of GMS / GMSD w.r.t. the inputs, one launch, no scratch.  The
 * reference differentiates its portable torch path instead
 * (functional.py:925-971).  x, y: float32 contiguous [N, C, H, W] (channels
 * pooled per image, as in the forward); mean / std_: the forward's per-image
 * GMS and GMSD (device, [N] float64); g_mean / g_std: d loss / d those
 * (device, [N] float64, either may be NULL).  dx / dy: [N, C, H, W] float32,
 * nullable (not both); positions the 2x2 pool drops (an odd last row or
 * column) are not written -- zero them first. */
FA_B200_API int fa_b200_gmsd_backward(const float* x, const float* y, int N,
                                      int C, int H, int W, int downsample,
                                      double T, double eps,
                                      const double* g_mean, const double* g_std,
                                      const double* mean, const double* std_,
                                      float* dx, float* dy, int device,
                                      void* stream);

/* Gradient of a pixel reduction (mse / l1 / charbonnier / huber) w.r.t. its
 * inputs.  Replaces the torch autograd the reference uses for these
 * (functional.py:1097-1141).  x, y: float32 contiguous [N, C, H, W];
 * g: device float64, [N] when per_image else [1] (d loss / d output);
 * luma as for fa_b200_pixel_reduce.  dx / dy nullable (not both). */
FA_B200_API int fa_b200_pixel_backward(const float* x, const float* y, int N,
                                       int C, int H, int W, const double* luma,
                                       int op, double param, const double* g,
                                       int per_image, float* dx, float* dy,
                                       int device, void* stream);

/* 2x2 mean pooling between MS-SSIM scales: out[n, c, i, j] = mean of the
 * 2x2 block x[n, c, 2i:2i+2, 2j:2j+2], an odd last row / column dropped
 * (F.avg_pool2d(x, 2)).  Replaces the reference's cast-then-pool
 * (functional.py:717-725, used at :885 and :930) by one pass over x in its
 * own dtype and strides.  luma (4 host doubles, nullable) projects RGB to
 * one channel first, as for fa_b200_pixel_reduce.  out: float32 contiguous
 * [N, C', H/2, W/2].  H and W must be at least 2. */
FA_B200_API int fa_b200_pool2(const fa_view* x, const double* luma, float* out,
                              int device, void* stream);

/* MATLAB ssim.m's automatic downsample (the reference's _matlab_downsample,
 * functional.py:575-586, torch pad + conv2d + strided slice): an f x f box
 * mean with replicated borders (pad f/2), sampled every f-th row and column.
 * out: float32 contiguous [N, C', ceil((H + 2(f/2) - f + 1)/f),
 * ceil((W + 2(f/2) - f + 1)/f)]; luma as for fa_b200_pool2.  2 <= f <= 64. */
FA_B200_API int fa_b200_box_downsample(const fa_view* x, const double* luma,
                                       int f, float* out, int device,
                                       void* stream);

/* Adjoint of fa_b200_box_downsample (no luma): g float32 [N, C, Ho, Wo] ->
 * dx float32 [N, C, H, W], every element written; border samples collect
 * the weight of each replicated copy. */
FA_B200_API int fa_b200_box_downsample_backward(const float* g, int N, int C,
                                                int H, int W, int f, float* dx,
                                                int device, void* stream);

/* Adjoint of fa_b200_pool2 (no luma): dx[n, c, h, w] = g[n, c, h/2, w/2] / 4,
 * zero on a dropped odd row / column.  g: float32 [N, C, H/2, W/2];
 * dx: float32 [N, C, H, W], every element written. */
FA_B200_API int fa_b200_pool2_backward(const float* g, int N, int C, int H,
                                       int W, float* dx, int device,
                                       void* stream);

/* A pixel loss (FA_OP_MSE / L1 / CHARB / HUBER) and its gradient from one
 * read of x and y, for training.  No single counterpart in the reference,
 * which reduces with fa_cuda_pixel_reduce (fa_cuda.cu:1078-1156) and
 * differentiates with torch autograd (functional.py:1097-1141), reading the
 * inputs again.  x, y: contiguous float32 [N, per_image_elems].  Outputs as
 * fa_b200_pixel_reduce (out_per_image [N] / out_total, nullable) and dx / dy
 * (nullable, not both) = the gradient, for an upstream gradient of 1, of the
 * batch mean (per_image = 0) or of each image's mean (per_image = 1).  The
 * workspace is sized by fa_b200_pixel_workspace_bytes. */
FA_B200_API int fa_b200_pixel_loss_grad(const float* x, const float* y, int N,
                                        long long per_image_elems, int op,
                                        double param, int per_image,
                                        void* workspace, size_t workspace_bytes,
                                        double* out_per_image, double* out_total,
                                        float* dx, float* dy, int device,
                                        void* stream);

/* Pixel reduction for callers that cannot allocate device memory.  No
 * counterpart in the reference: its reductions always take caller-allocated
 * scratch.  Callers such as host-application plugins that only receive frame
 * buffers, or code running where cudaMalloc is unavailable, can use this
 * variant: its scratch is a fixed array of FA_B200_NOALLOC_SCRATCH_BYTES
 * that lives in the library (held on every GPU that loads it until exit), so
 * the call allocates nothing.  Same arguments and outputs as
 * fa_b200_pixel_reduce minus the workspace.  Batches of more than
 * FA_B200_NOALLOC_MAX_IMAGES images return FA_E_SHAPE.  All calls on a
 * device share the array: calls that may overlap on the GPU race, so
 * serialise them.  The first call on a device (and the first in each new context of it, e.g.
 * after cudaDeviceReset) looks up the array's address;
 * make it before any stream capture. */
#define FA_B200_NOALLOC_SCRATCH_BYTES (64 * 1024)
#define FA_B200_NOALLOC_MAX_IMAGES 4096
FA_B200_API int fa_b200_pixel_reduce_noalloc(
    const fa_view* a, const fa_view* b, const double* luma, int op,
    double param, double psnr_bias, double* out_per_image, double* out_total,
    double* out_psnr_per_image, double* out_psnr_total,
    uint64_t* out_isum_per_image, int device, void* stream);

/* ----------------------------------------------------------------------- */
/* float64 block.  No native counterpart in the reference: its native SSIM /  */
/* MS-SSIM / GMSD decline float64 input (backend.py:466, 602) and run the     */
/* float64 torch path (functional.py:589-689, 697-901, 974-1082).  These      */
/* calls keep every moment, sum and gradient in double.  dtype must be        */
/* FA_F64; taps_host are the K double taps in HOST memory; the workspace      */
/* (sized by the *_workspace_bytes query) needs no zeroing (each call clears  */
/* its counters on `stream`).                                                 */
/* ----------------------------------------------------------------------- */

/* SSIM of float64 frames (reference.py:118-160 in float64): outputs as
 * fa_b200_ssim, the map as float64 [N, C', Hout, Wout]. */
FA_B200_API int fa_b200_ssim64_workspace_bytes(int n, int c, int h, int w, int K,
                                               int luma, size_t* out_bytes);
FA_B200_API int fa_b200_ssim64(const fa_view* x, const fa_view* y, const double* luma,
                               const double* taps_host, int K, double C1, double C2,
                               void* workspace, size_t workspace_bytes, double* map_out,
                               double* out_plane_s, double* out_plane_cs,
                               double* out_per_image, double* out_total, int device,
                               void* stream);
/* Gradient of the float64 SSIM: exactly one of dL_dmap ([N*C, Hout, Wout]),
 * grad_scalar ([1], of the batch mean) or gs + gcs ([N*C], of the per-plane
 * mean SSIM and cs) is given.  coef: caller scratch of 4*N*C*Hout*Wout
 * doubles.  x, y, dx, dy: contiguous [N, C, H, W] float64. */
FA_B200_API int fa_b200_ssim64_backward(const double* x, const double* y, int N, int C,
                                        int H, int W, const double* taps_host, int K,
                                        double C1, double C2, const double* dL_dmap,
                                        const double* grad_scalar, const double* gs,
                                        const double* gcs, double* coef, double* dx,
                                        double* dy, int device, void* stream);
/* 2x2 average pool of contiguous float64 planes (odd trailing row / column
 * dropped, reference.py:231-241) and its adjoint. */
FA_B200_API int fa_b200_pool64(const double* in, int NC, int H, int W, double* out,
                               int device, void* stream);
FA_B200_API int fa_b200_pool64_backward(const double* g, int NC, int H, int W,
                                        double* dx, int device, void* stream);
/* GMS mean / GMSD per image of float64 frames, as fa_b200_gmsd (map float64). */
FA_B200_API int fa_b200_gmsd64_workspace_bytes(int n, int c, int h, int w, int downsample,
                                               int luma, int device, size_t* out_bytes);
FA_B200_API int fa_b200_gmsd64(const fa_view* x, const fa_view* y, const double* luma,
                               double T, double eps, int downsample, void* workspace,
                               size_t workspace_bytes, double* map_out, double* out_mean,
                               double* out_std, int device, void* stream);
/* Gradient of the per-image (mean, std) of q for upstream g_mean, g_std [N],
 * given the forward's mean and std [N].  coef: caller scratch of
 * 4*N*C*Hout*Wout doubles (the GMS map size).  Contiguous float64 frames. */
FA_B200_API int fa_b200_gmsd64_backward(const double* x, const double* y, int N, int C,
                                        int H, int W, int downsample, double T, double eps,
                                        const double* g_mean, const double* g_std,
                                        const double* mean, const double* std_,
                                        double* coef, double* dx, double* dy, int device,
                                        void* stream);

/* SSIMULACRA 2 (replaces the reference's torch pipeline frame_analytics/
 * ssimulacra2.py:465-590, whose float64 transcription is reference.py:
 * 540-700).  x (original) and y (distorted): (N, 3, H, W) sRGB in
 * [0, data_range], any dtype and strides (stride_c = 0 replicates a gray
 * plane), H, W >= 8.  f64 = 0 computes colour, blur and maps in float (the
 * reference's default), 1 in double; sums are double either way.  weights:
 * the 108 Msssim::Score weights in HOST memory.  Outputs: per-image score [N]
 * and batch mean (nullable).  The workspace (size from the query; holds the
 * pyramid's linear planes) needs no zeroing. */
FA_B200_API int fa_b200_ssimulacra2_workspace_bytes(int n, int h, int w, int f64,
                                                    size_t* out_bytes);
FA_B200_API int fa_b200_ssimulacra2(const fa_view* x, const fa_view* y, double data_range,
                                    int f64, const double* weights, void* workspace,
                                    size_t workspace_bytes, double* out_per_image,
                                    double* out_total, int device, void* stream);

/* No counterpart in the reference: test hook of the bounded device-side
 * waits.  Launches one thread that waits `limit_ns` (at most 1 s) for an
 * mbarrier phase that nothing completes and then records FA_E_TIMEOUT the
 * way a staging wait that gave up does; nothing is copied, so nothing is left
 * in flight.  Returns FA_OK; the next compute call after the kernel has
 * finished returns FA_E_TIMEOUT. */
FA_B200_API int fa_b200_wait_selftest(unsigned long long limit_ns, int device, void* stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* FA_B200_H */
