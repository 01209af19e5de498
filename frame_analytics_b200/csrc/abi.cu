// extern "C" boundary of libfa_b200.so.  Every entry point validates its
// arguments on the host, sets the device, and enqueues on the caller's stream;
// none allocates and none synchronises.
#include "ssim_common.cuh"  // mbarrier helpers of the wait self-test

#include <algorithm>
#include <mutex>
#include <utility>
#include <array>
#include <atomic>
#include <cstring>

namespace fab {

int pixel_reduce_impl(const View& a, const View& b, int dtype, const double* luma, int op,
                      double param, double psnr_bias, void* ws, size_t ws_bytes,
                      double* out_pi, double* out_tot, double* out_ppi, double* out_ptot,
                      unsigned long long* out_isum, int device, cudaStream_t st);
size_t pixel_ws_bytes(int n_images, int device);
int ssim_fwd_impl(const View& x, const View& y, int dtype, const double* luma, const float* win,
                  int K, double shift, double C1, double C2, float* map_out, void* ws,
                  size_t ws_bytes, double* out_plane_s, double* out_plane_cs,
                  double* out_per_image, double* out_total, int device, cudaStream_t st,
                  const SqOut* sq = nullptr, const float* wdev = nullptr,
                  const GmOut* gm = nullptr);
bool ssim_gmsd_fusable(const View& x, const View& y, int dtype, int K, int device);
size_t ssim64_ws_bytes(int planes, int h, int w, int K);
int ssim64_fwd_impl(const View& x, const View& y, int dtype, const double* luma,
                    const double* taps, int K, double C1, double C2, void* ws, size_t ws_bytes,
                    double* map, double* out_plane_s, double* out_plane_cs,
                    double* out_per_image, double* out_total, cudaStream_t st);
int ssim64_bwd_impl(const double* x, const double* y, int N, int C, int H, int W,
                    const double* taps, int K, double C1, double C2, const double* dmap,
                    const double* gscalar, const double* gs, const double* gcs, double* coef,
                    double* dx, double* dy, cudaStream_t st);
int pool64_impl(const double* in, int NC, int H, int W, double* out, int device,
                cudaStream_t st);
int pool64_bwd_impl(const double* g, int NC, int H, int W, double* dx, int device,
                    cudaStream_t st);
size_t gmsd64_ws_bytes(int planes, int h, int w, int down, int device);
size_t su2_ws_bytes(int N, int H, int W, int fsize);
int su2_impl(const View& x, const View& y, int dtype, double data_range, int f64,
             const double* weights, void* ws, size_t ws_bytes, double* out_per_image,
             double* out_total, int device, cudaStream_t st);
int gmsd64_impl(const View& x, const View& y, int dtype, const double* luma, double T,
                double eps, int down, void* ws, size_t ws_bytes, double* map,
                double* out_mean, double* out_std, int device, cudaStream_t st);
int gmsd64_bwd_impl(const double* x, const double* y, int N, int C, int H, int W, int down,
                    double T, double eps, const double* gm, const double* gsd, const double* mu,
                    const double* sd, double* coef, double* dx, double* dy, int device,
                    cudaStream_t st);
size_t ssim_ws_bytes(int planes, int Hout, int Wout, int K, int device);
int ssim_bwd_impl(const float* x, const float* y, int N, int C, int H, int W, const float* win,
                  int K, double shift, double C1, double C2, const float* dmap,
                  const float* gscalar, const float* gs, const float* gcs, float* dx, float* dy,
                  int device, cudaStream_t st, const float* wdev = nullptr);
int gmsd_impl(const View& x, const View& y, int dtype, const double* luma, double T, double eps,
              int down, void* ws, size_t ws_bytes, float* map_out, double* out_mean,
              double* out_std, int device, cudaStream_t st);
int pixel_backward_impl(const float* x, const float* y, int N, int C, int H, int W,
                        const double* luma, int op, double param, const double* g,
                        int per_image, float* dx, float* dy, int device, cudaStream_t st);
size_t gmsd_ws_bytes(int planes, int h, int w, int down, int device);
int gmsd_backward_impl(const float* x, const float* y, int N, int C, int H, int W, int down,
                       double T, double eps, const double* gm, const double* gsd,
                       const double* mu, const double* sd, float* dx, float* dy, int device,
                       cudaStream_t st);

size_t ssim_loss_grad_ws_bytes(int N, int C, int H, int W, int K, int device);
int ssim_loss_grad_impl(const float* x, const float* y, int N, int C, int H, int W,
                        const float* taps, int K, double shift, double C1, double C2,
                        double upstream, void* ws,
                        size_t ws_bytes, double* out_plane_s, double* out_per_image,
                        double* out_total, float* dx, float* dy, int device, cudaStream_t st);
int grad_scale_impl(const float* in, long long per_image, int n, const double* s,
                    int per_image_scale, double mult, float* out, int device, cudaStream_t st);
int pixel_loss_grad_impl(const float* x, const float* y, int N, long long per, int op,
                         double param, int per_image, void* ws, size_t ws_bytes,
                         double* out_per_image, double* out_total, float* dx, float* dy,
                         int device, cudaStream_t st);
int pool2_impl(const View& x, int dtype, const double* luma, float* out, int device,
               cudaStream_t st);
int box_down_impl(const View& x, int dtype, const double* luma, int f, float* out, int device,
                  cudaStream_t st);
int box_down_backward_impl(const float* g, int N, int C, int H, int W, int f, float* dx,
                           int device, cudaStream_t st);
int pool2_backward_impl(const float* g, int N, int C, int H, int W, float* dx, int device,
                        cudaStream_t st);

// The multiprocessor count sizes every grid; cudaDeviceGetAttribute costs
// microseconds, so it is read once per device.
int sm_count(int device) {
  constexpr int MAXD = 64;
  static int cache[MAXD] = {0};
  if (device < 0) {
    if (cudaGetDevice(&device) != cudaSuccess) device = 0;
  }
  if (device < MAXD && cache[device] > 0) return cache[device];
  int v = 0;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || v <= 0)
    v = 148;
  if (device < MAXD) cache[device] = v;
  return v;
}

static View contiguous_view(const void* p, int n, int c, int h, int w) {
  View v;
  v.data = p;
  v.n = n; v.c = c; v.h = h; v.w = w;
  v.sh = w;
  v.sc = (long long)h * w;
  v.sn = (long long)c * h * w;
  return v;
}

static bool view_ok(const fa_view* v) {
  return v && v->data && v->w > 0 && v->h > 0 && v->c > 0 && v->n > 0;
}


// The bounded waits' error word.  Pinned, mapped host memory: the kernels
// store to it without a copy back, and the host reads it without a
// synchronisation.  It is allocated once per process by the first call that
// launches a waiting kernel.  If that call happens under stream capture, the
// thread's capture mode is relaxed for the allocation alone (a host
// allocation touches no stream).
static std::atomic<unsigned int*> g_wait_word{nullptr};

unsigned int* wait_error_word() {
  unsigned int* w = g_wait_word.load(std::memory_order_acquire);
  if (w) return w;
  static std::mutex mu;
  std::lock_guard<std::mutex> g(mu);
  w = g_wait_word.load(std::memory_order_acquire);
  if (w) return w;
  cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
  cudaThreadExchangeStreamCaptureMode(&mode);
  void* h = nullptr;
  const cudaError_t e = cudaHostAlloc(&h, 64, cudaHostAllocMapped | cudaHostAllocPortable);
  cudaThreadExchangeStreamCaptureMode(&mode);
  if (e != cudaSuccess) {
    cudaGetLastError();  // not sticky: the waits then only give up
    return nullptr;
  }
  void* d = nullptr;
  if (cudaHostGetDevicePointer(&d, h, 0) != cudaSuccess || d != h) {
    // every 64-bit CUDA platform has unified addressing; without it the word
    // stays unused rather than being read through the wrong address
    cudaGetLastError();
    cudaFreeHost(h);
    return nullptr;
  }
  std::memset(h, 0, 64);
  w = static_cast<unsigned int*>(h);
  g_wait_word.store(w, std::memory_order_release);
  return w;
}

int take_wait_error() {
  unsigned int* w = g_wait_word.load(std::memory_order_acquire);
  if (!w) return FA_OK;
  if (__atomic_load_n(w, __ATOMIC_ACQUIRE) == 0u) return FA_OK;
  const unsigned v = __atomic_exchange_n(w, 0u, __ATOMIC_ACQ_REL);
  return v ? FA_E_TIMEOUT : FA_OK;
}

// A wait on an mbarrier phase that nothing completes: no copy is in flight,
// so the only effect of running out of time is the error word.
__global__ void wait_selftest_kernel(unsigned* err, unsigned long long limit_ns) {
  __shared__ __align__(8) unsigned long long bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_async_smem();
    mbar_wait_slow(smem_u32(&bar), 0u, err, limit_ns);
  }
}

}  // namespace fab

using namespace fab;

extern "C" {

// ---------------------------------------------------------------------------
// reference-compatible block
// ---------------------------------------------------------------------------

FA_B200_API int fa_cuda_abi_version(void) { return FA_ABI_VERSION; }

FA_B200_API const char* fa_cuda_error_string(int code) {
  if (code < 0) return cudaGetErrorString(static_cast<cudaError_t>(-code));
  switch (code) {
    case FA_OK: return "ok";
    case FA_E_DTYPE: return "unsupported dtype";
    case FA_E_SHAPE: return "unsupported shape";
    case FA_E_WINDOW: return "unsupported window size";
    case FA_E_OP: return "unknown pixel op";
    case FA_E_ARG: return "invalid argument";
    case FA_E_NOCUDA: return "no CUDA device";
    case FA_E_TIMEOUT: return "a device-side wait timed out; the results of the kernel that waited are invalid";
    default: return "internal error";
  }
}

FA_B200_API int fa_cuda_device_count(int* out_count) {
  int n = 0;
  const cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) {
    if (out_count) *out_count = 0;
    return -static_cast<int>(e);
  }
  if (out_count) *out_count = n;
  return FA_OK;
}

FA_B200_API int fa_cuda_pixel_workspace(int64_t n_images, int64_t n_per_image, int device,
                                        int* out_bpi) {
  if (!out_bpi) return FA_E_ARG;
  if (n_images <= 0 || n_per_image <= 0 || n_images > INT32_MAX) return FA_E_SHAPE;
  const size_t bytes = pixel_ws_bytes((int)n_images, device);
  const size_t row = (size_t)n_images * 8;
  *out_bpi = (int)((bytes + row - 1) / row);
  return FA_OK;
}

FA_B200_API int fa_cuda_pixel_reduce(const void* a, const void* b, int dtype, int64_t n_images,
                                     int64_t n_per_image, int op, double param,
                                     double psnr_bias, double* partial, int bpi,
                                     double* out_per_image, double* out_total,
                                     double* out_psnr_per_image, double* out_psnr_total,
                                     int device, void* stream) {
  FAB_PENDING();
  if (!a || !b || !partial) return FA_E_ARG;
  if (op < 0 || op > 3) return FA_E_OP;
  if (n_images <= 0 || n_per_image <= 0 || bpi <= 0 || n_images > INT32_MAX ||
      n_per_image > INT32_MAX)
    return FA_E_SHAPE;
  FAB_DEVICE_SCOPE(device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // the caller's scratch comes from torch.empty: clear the counters
  FAB_TRY(cudaMemsetAsync(partial, 0, FAB_COUNTER_BYTES, st));
  View va = contiguous_view(a, (int)n_images, 1, 1, (int)n_per_image);
  View vb = contiguous_view(b, (int)n_images, 1, 1, (int)n_per_image);
  return pixel_reduce_impl(va, vb, dtype, nullptr, op, param, psnr_bias, partial,
                           (size_t)n_images * bpi * 8, out_per_image, out_total,
                           out_psnr_per_image, out_psnr_total, nullptr, device, st);
}

FA_B200_API int fa_cuda_ssim_workspace(int H, int W, int K, int* out_bpp) {
  if (!out_bpp) return FA_E_ARG;
  if (K < 3 || K > FA_MAX_WIN || (K & 1) == 0) return FA_E_WINDOW;
  const int Hout = H - K + 1, Wout = W - K + 1;
  if (Hout <= 0 || Wout <= 0) return FA_E_SHAPE;
  // per plane: two partial arrays at the most-chunked plan (one plane), plus
  // the counter block spread over planes
  const size_t per_plane = ssim_ws_bytes(1, Hout, Wout, K, -1);
  *out_bpp = (int)((per_plane + 7) / 8);
  return FA_OK;
}

FA_B200_API int fa_cuda_ssim(const void* x, const void* y, int dtype, int N, int C, int H, int W,
                             const float* win, int K, double shift, double C1, double C2,
                             float* map_out, double* partial, int bpp, double* out_per_image,
                             double* out_total, int device, void* stream) {
  FAB_PENDING();
  if (!x || !y || !win || !partial) return FA_E_ARG;
  if (N <= 0 || C <= 0 || H <= 0 || W <= 0 || bpp <= 0) return FA_E_SHAPE;
  FAB_DEVICE_SCOPE(device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (K < 3 || K > FA_MAX_WIN || (K & 1) == 0) return FA_E_WINDOW;
  FAB_TRY(cudaMemsetAsync(partial, 0, FAB_COUNTER_BYTES, st));
  View vx = contiguous_view(x, N, C, H, W), vy = contiguous_view(y, N, C, H, W);
  // the taps stay on the device: the kernel reads `win` itself
  return ssim_fwd_impl(vx, vy, dtype, nullptr, nullptr, K, shift, C1, C2, map_out, partial,
                       (size_t)N * C * bpp * 8, nullptr, nullptr, out_per_image, out_total,
                       device, st, nullptr, win);
}

FA_B200_API int fa_cuda_ssim_cs(const void* x, const void* y, int dtype, int N, int C, int H,
                                int W, const float* win, int K, double shift, double C1,
                                double C2, double* partial, double* partial_cs, int bpp,
                                double* out_s, double* out_cs, int device, void* stream) {
  FAB_PENDING();
  if (!x || !y || !win || !partial || !partial_cs || !out_s || !out_cs) return FA_E_ARG;
  if (N <= 0 || C <= 0 || H <= 0 || W <= 0 || bpp <= 0) return FA_E_SHAPE;
  FAB_DEVICE_SCOPE(device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (K < 3 || K > FA_MAX_WIN || (K & 1) == 0) return FA_E_WINDOW;
  FAB_TRY(cudaMemsetAsync(partial, 0, FAB_COUNTER_BYTES, st));
  View vx = contiguous_view(x, N, C, H, W), vy = contiguous_view(y, N, C, H, W);
  return ssim_fwd_impl(vx, vy, dtype, nullptr, nullptr, K, shift, C1, C2, nullptr, partial,
                       (size_t)N * C * bpp * 8, out_s, out_cs, nullptr, nullptr, device, st,
                       nullptr, win);
}

FA_B200_API int fa_cuda_ssim_backward(const float* x, const float* y, const float* dL_dmap,
                                      const float* grad_scalar, const float* win, int K, int N,
                                      int C, int H, int W, double shift, double C1, double C2,
                                      float* aux, float* dx, float* dy, int device,
                                      void* stream) {
  FAB_PENDING();
  (void)aux;
  if (dL_dmap && grad_scalar) grad_scalar = nullptr;  // the map wins, as in the reference
  if (!win) return FA_E_ARG;
  if (K < 3 || K > FA_MAX_WIN || (K & 1) == 0) return FA_E_WINDOW;
  FAB_DEVICE_SCOPE(device);
  return ssim_bwd_impl(x, y, N, C, H, W, nullptr, K, shift, C1, C2, dL_dmap, grad_scalar,
                       nullptr, nullptr, dx, dy, device, static_cast<cudaStream_t>(stream), win);
}

FA_B200_API int fa_cuda_ssim_cs_backward(const float* x, const float* y, const float* gs,
                                         const float* gcs, const float* win, int K, int N, int C,
                                         int H, int W, double shift, double C1, double C2,
                                         float* aux, float* dx, float* dy, int device,
                                         void* stream) {
  FAB_PENDING();
  (void)aux;
  if (!gs || !gcs || !win) return FA_E_ARG;
  if (K < 3 || K > FA_MAX_WIN || (K & 1) == 0) return FA_E_WINDOW;
  FAB_DEVICE_SCOPE(device);
  return ssim_bwd_impl(x, y, N, C, H, W, nullptr, K, shift, C1, C2, nullptr, nullptr, gs, gcs,
                       dx, dy, device, static_cast<cudaStream_t>(stream), win);
}

FA_B200_API int fa_cuda_gmsd_workspace(int H, int W, int downsample, int* out_bpp) {
  if (!out_bpp) return FA_E_ARG;
  if (H <= 0 || W <= 0) return FA_E_SHAPE;
  const int hd = downsample ? H / 2 : H, wd = downsample ? W / 2 : W;
  if (hd < 3 || wd < 3) return FA_E_SHAPE;
  const size_t per_plane = gmsd_ws_bytes(1, H, W, downsample, -1);
  *out_bpp = (int)((per_plane + 7) / 8);
  return FA_OK;
}

FA_B200_API int fa_cuda_gmsd(const void* x, const void* y, int dtype, int N, int C, int H, int W,
                             double Tc, double eps, int downsample, double* psum,
                             double* psumsq, int bpp, double* out_mean, double* out_std,
                             int device, void* stream) {
  FAB_PENDING();
  (void)psumsq;
  if (!x || !y || !psum || !out_mean || !out_std) return FA_E_ARG;
  if (N <= 0 || C <= 0 || H <= 0 || W <= 0 || bpp <= 0) return FA_E_SHAPE;
  FAB_DEVICE_SCOPE(device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  FAB_TRY(cudaMemsetAsync(psum, 0, FAB_COUNTER_BYTES, st));
  View vx = contiguous_view(x, N, C, H, W), vy = contiguous_view(y, N, C, H, W);
  return gmsd_impl(vx, vy, dtype, nullptr, Tc, eps, downsample, psum, (size_t)N * C * bpp * 8,
                   nullptr, out_mean, out_std, device, st);
}

// ---------------------------------------------------------------------------
// extended block
// ---------------------------------------------------------------------------

FA_B200_API int fa_b200_abi_version(void) { return FA_B200_ABI_VERSION; }

FA_B200_API int fa_b200_pixel_workspace_bytes(int n_images, int device, size_t* out_bytes) {
  if (!out_bytes) return FA_E_ARG;
  if (n_images <= 0) return FA_E_SHAPE;
  *out_bytes = pixel_ws_bytes(n_images, device);
  return FA_OK;
}

FA_B200_API int fa_b200_pixel_reduce(const fa_view* a, const fa_view* b, const double* luma,
                                     int op, double param, double psnr_bias, void* workspace,
                                     size_t workspace_bytes, double* out_per_image,
                                     double* out_total, double* out_psnr_per_image,
                                     double* out_psnr_total, uint64_t* out_isum_per_image,
                                     int device, void* stream) {
  FAB_PENDING();
  if (!view_ok(a) || !view_ok(b)) return FA_E_ARG;
  if (a->dtype != b->dtype) return FA_E_DTYPE;
  FAB_DEVICE_SCOPE(device);
  return pixel_reduce_impl(to_view(*a), to_view(*b), a->dtype, luma, op, param, psnr_bias,
                           workspace, workspace_bytes, out_per_image, out_total,
                           out_psnr_per_image, out_psnr_total,
                           reinterpret_cast<unsigned long long*>(out_isum_per_image), device,
                           static_cast<cudaStream_t>(stream));
}

FA_B200_API int fa_b200_ssim_workspace_bytes(int n, int c, int h, int w, int K, int device,
                                             size_t* out_bytes) {
  if (!out_bytes) return FA_E_ARG;
  if (K < 3 || K > FA_MAX_WIN || (K & 1) == 0) return FA_E_WINDOW;
  if (n <= 0 || c <= 0 || h - K + 1 <= 0 || w - K + 1 <= 0) return FA_E_SHAPE;
  *out_bytes = ssim_ws_bytes(n * c, h - K + 1, w - K + 1, K, device);
  return FA_OK;
}

FA_B200_API int fa_b200_ssim(const fa_view* x, const fa_view* y, const double* luma,
                             const float* win, int K, double shift, double C1, double C2,
                             float* map_out, void* workspace, size_t workspace_bytes,
                             double* out_plane_s, double* out_plane_cs, double* out_per_image,
                             double* out_total, int device, void* stream) {
  FAB_PENDING();
  if (!view_ok(x) || !view_ok(y)) return FA_E_ARG;
  if (x->dtype != y->dtype) return FA_E_DTYPE;
  FAB_DEVICE_SCOPE(device);
  return ssim_fwd_impl(to_view(*x), to_view(*y), x->dtype, luma, win, K, shift, C1, C2, map_out,
                       workspace, workspace_bytes, out_plane_s, out_plane_cs, out_per_image,
                       out_total, device, static_cast<cudaStream_t>(stream));
}

FA_B200_API int fa_b200_ssim_backward(const float* x, const float* y, int N, int C, int H, int W,
                                      const float* win, int K, double shift, double C1,
                                      double C2, const float* dL_dmap, const float* g_scalar,
                                      const float* gs, const float* gcs, float* dx, float* dy,
                                      int device, void* stream) {
  FAB_PENDING();
  FAB_DEVICE_SCOPE(device);
  return ssim_bwd_impl(x, y, N, C, H, W, win, K, shift, C1, C2, dL_dmap, g_scalar, gs, gcs, dx,
                       dy, device, static_cast<cudaStream_t>(stream));
}

FA_B200_API int fa_b200_ssim_mse(const fa_view* x, const fa_view* y, const float* win, int K,
                                 double shift, double C1, double C2, double psnr_bias,
                                 void* workspace, size_t workspace_bytes, double* out_plane_s,
                                 double* out_per_image, double* out_total,
                                 double* out_mse_per_image, double* out_mse_total,
                                 double* out_psnr_per_image, double* out_psnr_total,
                                 uint64_t* out_ssd_per_image, int device, void* stream) {
  FAB_PENDING();
  if (!view_ok(x) || !view_ok(y)) return FA_E_ARG;
  if (x->dtype != y->dtype) return FA_E_DTYPE;
  FAB_DEVICE_SCOPE(device);
  const SqOut sq{psnr_bias, out_mse_per_image, out_mse_total, out_psnr_per_image,
                 out_psnr_total, reinterpret_cast<unsigned long long*>(out_ssd_per_image)};
  return ssim_fwd_impl(to_view(*x), to_view(*y), x->dtype, nullptr, win, K, shift, C1, C2,
                       nullptr, workspace, workspace_bytes, out_plane_s, nullptr, out_per_image,
                       out_total, device, static_cast<cudaStream_t>(stream), &sq);
}

FA_B200_API int fa_b200_ssim_gmsd_fusable(const fa_view* x, const fa_view* y, int K,
                                          int device, int* out_ok) {
  if (!out_ok) return FA_E_ARG;
  *out_ok = 0;
  if (!view_ok(x) || !view_ok(y)) return FA_E_ARG;
  if (x->dtype != y->dtype) return FA_E_DTYPE;
  FAB_DEVICE_SCOPE(device);
  *out_ok = ssim_gmsd_fusable(to_view(*x), to_view(*y), x->dtype, K, device) ? 1 : 0;
  return FA_OK;
}

FA_B200_API int fa_b200_ssim_gmsd(const fa_view* x, const fa_view* y, const float* win, int K,
                                  double shift, double C1, double C2, double gmsd_T,
                                  double gmsd_eps, double psnr_bias, void* workspace,
                                  size_t workspace_bytes, double* out_plane_s,
                                  double* out_per_image, double* out_total,
                                  double* out_gms_per_image, double* out_gmsd_per_image,
                                  double* out_mse_per_image, double* out_mse_total,
                                  double* out_psnr_per_image, double* out_psnr_total,
                                  uint64_t* out_ssd_per_image, int device, void* stream) {
  FAB_PENDING();
  if (!view_ok(x) || !view_ok(y)) return FA_E_ARG;
  if (x->dtype != y->dtype) return FA_E_DTYPE;
  FAB_DEVICE_SCOPE(device);
  const SqOut sq{psnr_bias, out_mse_per_image, out_mse_total, out_psnr_per_image,
                 out_psnr_total, reinterpret_cast<unsigned long long*>(out_ssd_per_image)};
  const bool want_sq = out_mse_per_image || out_mse_total || out_psnr_per_image ||
                       out_psnr_total || out_ssd_per_image;
  const GmOut gm{gmsd_T, gmsd_eps, out_gms_per_image, out_gmsd_per_image};
  return ssim_fwd_impl(to_view(*x), to_view(*y), x->dtype, nullptr, win, K, shift, C1, C2,
                       nullptr, workspace, workspace_bytes, out_plane_s, nullptr, out_per_image,
                       out_total, device, static_cast<cudaStream_t>(stream),
                       want_sq ? &sq : nullptr, nullptr, &gm);
}

FA_B200_API int fa_b200_ssim_loss_grad_workspace_bytes(int n, int c, int h, int w, int K,
                                                       int device, size_t* out_bytes) {
  if (!out_bytes) return FA_E_ARG;
  if (K < 3 || K > FA_MAX_WIN || (K & 1) == 0) return FA_E_WINDOW;
  if (n <= 0 || c <= 0 || h - K + 1 <= 0 || w - K + 1 <= 0) return FA_E_SHAPE;
  *out_bytes = ssim_loss_grad_ws_bytes(n, c, h, w, K, device);
  return FA_OK;
}

FA_B200_API int fa_b200_ssim_loss_grad(const float* x, const float* y, int N, int C, int H, int W,
                                       const float* win, int K, double shift, double C1,
                                       double C2, double upstream, void* workspace,
                                       size_t workspace_bytes, double* out_plane_s,
                                       double* out_per_image, double* out_total, float* dx,
                                       float* dy, int device, void* stream) {
  FAB_PENDING();
  FAB_DEVICE_SCOPE(device);
  return ssim_loss_grad_impl(x, y, N, C, H, W, win, K, shift, C1, C2, upstream, workspace,
                             workspace_bytes,
                             out_plane_s, out_per_image, out_total, dx, dy, device,
                             static_cast<cudaStream_t>(stream));
}

FA_B200_API int fa_b200_gmsd_workspace_bytes(int n, int c, int h, int w, int downsample,
                                             int device, size_t* out_bytes) {
  if (!out_bytes) return FA_E_ARG;
  if (n <= 0 || c <= 0 || h <= 0 || w <= 0) return FA_E_SHAPE;
  const int hd = downsample ? h / 2 : h, wd = downsample ? w / 2 : w;
  if (hd < 3 || wd < 3) return FA_E_SHAPE;
  *out_bytes = gmsd_ws_bytes(n * c, h, w, downsample, device);
  return FA_OK;
}

FA_B200_API int fa_b200_gmsd(const fa_view* x, const fa_view* y, const double* luma, double T,
                             double eps, int downsample, void* workspace,
                             size_t workspace_bytes, float* map_out, double* out_mean,
                             double* out_std, int device, void* stream) {
  FAB_PENDING();
  if (!view_ok(x) || !view_ok(y)) return FA_E_ARG;
  if (x->dtype != y->dtype) return FA_E_DTYPE;
  FAB_DEVICE_SCOPE(device);
  return gmsd_impl(to_view(*x), to_view(*y), x->dtype, luma, T, eps, downsample, workspace,
                   workspace_bytes, map_out, out_mean, out_std, device,
                   static_cast<cudaStream_t>(stream));
}

FA_B200_API int fa_b200_gmsd_backward(const float* x, const float* y, int N, int C, int H,
                                      int W, int downsample, double T, double eps,
                                      const double* g_mean, const double* g_std,
                                      const double* mean, const double* std_, float* dx,
                                      float* dy, int device, void* stream) {
  FAB_PENDING();
  FAB_DEVICE_SCOPE(device);
  return gmsd_backward_impl(x, y, N, C, H, W, downsample, T, eps, g_mean, g_std, mean, std_, dx,
                            dy, device, static_cast<cudaStream_t>(stream));
}

FA_B200_API int fa_b200_pixel_backward(const float* x, const float* y, int N, int C, int H,
                                       int W, const double* luma, int op, double param,
                                       const double* g, int per_image, float* dx, float* dy,
                                       int device, void* stream) {
  FAB_PENDING();
  FAB_DEVICE_SCOPE(device);
  return pixel_backward_impl(x, y, N, C, H, W, luma, op, param, g, per_image, dx, dy, device,
                             static_cast<cudaStream_t>(stream));
}

FA_B200_API int fa_b200_pool2(const fa_view* x, const double* luma, float* out, int device,
                              void* stream) {
  FAB_PENDING();
  if (!view_ok(x) || !out) return FA_E_ARG;
  FAB_DEVICE_SCOPE(device);
  return pool2_impl(to_view(*x), x->dtype, luma, out, device, static_cast<cudaStream_t>(stream));
}

FA_B200_API int fa_b200_pool2_backward(const float* g, int N, int C, int H, int W, float* dx,
                                       int device, void* stream) {
  FAB_PENDING();
  FAB_DEVICE_SCOPE(device);
  return pool2_backward_impl(g, N, C, H, W, dx, device, static_cast<cudaStream_t>(stream));
}

FA_B200_API int fa_b200_grad_scale(const float* in, long long per_image, int n, const double* s,
                                   int per_image_scale, double mult, float* out, int device,
                                   void* stream) {
  FAB_PENDING();
  FAB_DEVICE_SCOPE(device);
  return grad_scale_impl(in, per_image, n, s, per_image_scale, mult, out, device,
                         static_cast<cudaStream_t>(stream));
}

FA_B200_API int fa_b200_box_downsample(const fa_view* x, const double* luma, int f, float* out,
                                       int device, void* stream) {
  FAB_PENDING();
  if (!view_ok(x) || !out) return FA_E_ARG;
  FAB_DEVICE_SCOPE(device);
  return box_down_impl(to_view(*x), x->dtype, luma, f, out, device,
                       static_cast<cudaStream_t>(stream));
}

FA_B200_API int fa_b200_box_downsample_backward(const float* g, int N, int C, int H, int W,
                                                int f, float* dx, int device, void* stream) {
  FAB_PENDING();
  FAB_DEVICE_SCOPE(device);
  return box_down_backward_impl(g, N, C, H, W, f, dx, device, static_cast<cudaStream_t>(stream));
}

FA_B200_API int fa_b200_pixel_loss_grad(const float* x, const float* y, int N,
                                        long long per_image_elems, int op, double param,
                                        int per_image, void* workspace, size_t workspace_bytes,
                                        double* out_per_image, double* out_total, float* dx,
                                        float* dy, int device, void* stream) {
  FAB_PENDING();
  FAB_DEVICE_SCOPE(device);
  return pixel_loss_grad_impl(x, y, N, per_image_elems, op, param, per_image, workspace,
                              workspace_bytes, out_per_image, out_total, dx, dy, device,
                              static_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------------------
// float64 block
// ---------------------------------------------------------------------------

FA_B200_API int fa_b200_ssim64_workspace_bytes(int n, int c, int h, int w, int K, int luma,
                                               size_t* out_bytes) {
  if (!out_bytes) return FA_E_ARG;
  if (n <= 0 || c <= 0 || h < K || w < K) return FA_E_SHAPE;
  *out_bytes = ssim64_ws_bytes(n * (luma ? 1 : c), h, w, K);
  return FA_OK;
}

FA_B200_API int fa_b200_ssim64(const fa_view* x, const fa_view* y, const double* luma,
                               const double* taps_host, int K, double C1, double C2,
                               void* workspace, size_t workspace_bytes, double* map_out,
                               double* out_plane_s, double* out_plane_cs, double* out_per_image,
                               double* out_total, int device, void* stream) {
  FAB_PENDING();
  if (!view_ok(x) || !view_ok(y)) return FA_E_ARG;
  if (x->dtype != y->dtype) return FA_E_DTYPE;
  FAB_DEVICE_SCOPE(device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (workspace) FAB_TRY(cudaMemsetAsync(workspace, 0, FAB_COUNTER_BYTES, st));
  return ssim64_fwd_impl(to_view(*x), to_view(*y), x->dtype, luma, taps_host, K, C1, C2,
                         workspace, workspace_bytes, map_out, out_plane_s, out_plane_cs,
                         out_per_image, out_total, st);
}

FA_B200_API int fa_b200_ssim64_backward(const double* x, const double* y, int N, int C, int H,
                                        int W, const double* taps_host, int K, double C1,
                                        double C2, const double* dL_dmap,
                                        const double* grad_scalar, const double* gs,
                                        const double* gcs, double* coef, double* dx,
                                        double* dy, int device, void* stream) {
  FAB_PENDING();
  FAB_DEVICE_SCOPE(device);
  return ssim64_bwd_impl(x, y, N, C, H, W, taps_host, K, C1, C2, dL_dmap, grad_scalar, gs, gcs,
                         coef, dx, dy, static_cast<cudaStream_t>(stream));
}

FA_B200_API int fa_b200_pool64(const double* in, int NC, int H, int W, double* out, int device,
                               void* stream) {
  FAB_PENDING();
  FAB_DEVICE_SCOPE(device);
  return pool64_impl(in, NC, H, W, out, device, static_cast<cudaStream_t>(stream));
}

FA_B200_API int fa_b200_pool64_backward(const double* g, int NC, int H, int W, double* dx,
                                        int device, void* stream) {
  FAB_PENDING();
  FAB_DEVICE_SCOPE(device);
  return pool64_bwd_impl(g, NC, H, W, dx, device, static_cast<cudaStream_t>(stream));
}

FA_B200_API int fa_b200_gmsd64_workspace_bytes(int n, int c, int h, int w, int downsample,
                                               int luma, int device, size_t* out_bytes) {
  if (!out_bytes) return FA_E_ARG;
  if (n <= 0 || c <= 0 || h <= 0 || w <= 0) return FA_E_SHAPE;
  FAB_DEVICE_SCOPE(device);
  *out_bytes = gmsd64_ws_bytes(n * (luma ? 1 : c), h, w, downsample, device);
  return FA_OK;
}

FA_B200_API int fa_b200_gmsd64(const fa_view* x, const fa_view* y, const double* luma, double T,
                               double eps, int downsample, void* workspace,
                               size_t workspace_bytes, double* map_out, double* out_mean,
                               double* out_std, int device, void* stream) {
  FAB_PENDING();
  if (!view_ok(x) || !view_ok(y)) return FA_E_ARG;
  if (x->dtype != y->dtype) return FA_E_DTYPE;
  FAB_DEVICE_SCOPE(device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (workspace) FAB_TRY(cudaMemsetAsync(workspace, 0, FAB_COUNTER_BYTES, st));
  return gmsd64_impl(to_view(*x), to_view(*y), x->dtype, luma, T, eps, downsample, workspace,
                     workspace_bytes, map_out, out_mean, out_std, device, st);
}

FA_B200_API int fa_b200_gmsd64_backward(const double* x, const double* y, int N, int C, int H,
                                        int W, int downsample, double T, double eps,
                                        const double* g_mean, const double* g_std,
                                        const double* mean, const double* std_, double* coef,
                                        double* dx, double* dy, int device, void* stream) {
  FAB_PENDING();
  FAB_DEVICE_SCOPE(device);
  return gmsd64_bwd_impl(x, y, N, C, H, W, downsample, T, eps, g_mean, g_std, mean, std_, coef,
                         dx, dy, device, static_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------------------
// SSIMULACRA 2
// ---------------------------------------------------------------------------

FA_B200_API int fa_b200_ssimulacra2_workspace_bytes(int n, int h, int w, int f64,
                                                    size_t* out_bytes) {
  if (!out_bytes) return FA_E_ARG;
  if (n <= 0 || h < 8 || w < 8) return FA_E_SHAPE;
  *out_bytes = su2_ws_bytes(n, h, w, f64 ? 8 : 4);
  return FA_OK;
}

FA_B200_API int fa_b200_ssimulacra2(const fa_view* x, const fa_view* y, double data_range,
                                    int f64, const double* weights, void* workspace,
                                    size_t workspace_bytes, double* out_per_image,
                                    double* out_total, int device, void* stream) {
  FAB_PENDING();
  if (!view_ok(x) || !view_ok(y)) return FA_E_ARG;
  if (x->dtype != y->dtype) return FA_E_DTYPE;
  FAB_DEVICE_SCOPE(device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (!workspace) return FA_E_ARG;
  FAB_TRY(cudaMemsetAsync(workspace, 0, FAB_COUNTER_BYTES, st));
  return su2_impl(to_view(*x), to_view(*y), x->dtype, data_range, f64, weights, workspace,
                  workspace_bytes, out_per_image, out_total, device, st);
}

// Test hook of the bounded waits: one thread waits `limit_ns` for an mbarrier
// phase that nothing completes, then records the time-out exactly as a
// staging wait that gave up would.  Nothing is copied and nothing is left in
// flight.  The next compute call returns FA_E_TIMEOUT.
FA_B200_API int fa_b200_wait_selftest(unsigned long long limit_ns, int device, void* stream) {
  FAB_PENDING();
  FAB_DEVICE_SCOPE(device);
  unsigned* w = wait_error_word();
  if (!w) return FA_E_INTERNAL;
  if (limit_ns > 1000000000ull) return FA_E_ARG;
  wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(w, limit_ns);
  FAB_LAUNCH_CHECK();
  return FA_OK;
}

}  // extern "C"
