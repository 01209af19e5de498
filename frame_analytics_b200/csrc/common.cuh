// Shared device/host helpers of the sm_100a metric kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <type_traits>

#include "../../include/fa_b200.h"

namespace fab {

// ---------------------------------------------------------------------------
// element types
// ---------------------------------------------------------------------------
struct f16_t { unsigned short bits; };
struct bf16_t { unsigned short bits; };

// Widening loads.  bf16 is the top half of an IEEE float; fp16 goes through
// the hardware conversion.  `getd` keeps float64 input wide (the reference
// narrows nothing it promised to keep: fa_cuda.cu:97-121).
template <typename T> struct Ld {
  static __device__ __forceinline__ float f(T v) { return static_cast<float>(v); }
  static __device__ __forceinline__ double d(T v) { return static_cast<double>(v); }
};
template <> struct Ld<f16_t> {
  static __device__ __forceinline__ float f(f16_t v) {
    return __half2float(__ushort_as_half(v.bits));
  }
  static __device__ __forceinline__ double d(f16_t v) { return (double)f(v); }
};
template <> struct Ld<bf16_t> {
  static __device__ __forceinline__ float f(bf16_t v) {
    return __uint_as_float(static_cast<unsigned>(v.bits) << 16);
  }
  static __device__ __forceinline__ double d(bf16_t v) { return (double)f(v); }
};

// Read-only scalar load through the non-coherent path.
template <typename T>
__device__ __forceinline__ T ldro(const T* p) {
  if constexpr (std::is_same<T, unsigned short>::value) {
    return __ldg(p);
  } else if constexpr (sizeof(T) == 2) {  // f16_t / bf16_t bit containers
    const unsigned short b = __ldg(reinterpret_cast<const unsigned short*>(p));
    T v;
    v.bits = b;
    return v;
  } else {
    return __ldg(p);
  }
}

// ---------------------------------------------------------------------------
// views
// ---------------------------------------------------------------------------
struct View {
  const void* data;
  int n, c, h, w;
  long long sn, sc, sh;
};

static inline View to_view(const fa_view& v) {
  View o;
  o.data = v.data;
  o.n = v.n; o.c = v.c; o.h = v.h; o.w = v.w;
  o.sn = v.stride_n; o.sc = v.stride_c; o.sh = v.stride_h;
  return o;
}

// Luma coefficients, already in the metric's units (offset * L in k3).
struct Luma {
  float k0, k1, k2, k3;
  double d0, d1, d2, d3;
  int on;
};

static inline Luma make_luma(const double* k) {
  Luma l{};
  if (k) {
    l.on = 1;
    l.d0 = k[0]; l.d1 = k[1]; l.d2 = k[2]; l.d3 = k[3];
    l.k0 = (float)k[0]; l.k1 = (float)k[1]; l.k2 = (float)k[2]; l.k3 = (float)k[3];
  }
  return l;
}

// ---------------------------------------------------------------------------
// reductions
// ---------------------------------------------------------------------------
template <typename A>
__device__ __forceinline__ A warp_sum(A v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide sum, result valid in every thread.  `sm` holds >= 32 A.
template <typename A>
__device__ __forceinline__ A block_sum(A v, A* sm) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) sm[wid] = v;
  __syncthreads();
  A r = A(0);
  for (int i = 0; i < nw; ++i) r += sm[i];  // fixed order: deterministic
  return r;
}

// Grid completion: every block calls this once after publishing its partial
// results.  Returns true in exactly one block (the last to arrive), after
// which all other blocks' partials are visible to it.  That block resets the
// counter, so the next launch on the same stream finds it at zero again.
__device__ __forceinline__ bool last_block_arrived(unsigned int* counter,
                                                   unsigned int nblocks,
                                                   int* s_flag) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned int t = atomicAdd(counter, 1u);
    const int last = (t == nblocks - 1);
    if (last) {
      *counter = 0u;
      __threadfence();
    }
    *s_flag = last;
  }
  __syncthreads();
  return *s_flag != 0;
}

// ---------------------------------------------------------------------------
// host plumbing
// ---------------------------------------------------------------------------
// Makes `dev` current for its lifetime and puts the caller's device back;
// dev < 0 keeps whatever is current.
class ScopedDevice {
 public:
  explicit ScopedDevice(int dev) : err_(cudaGetDevice(&saved_)) {
    if (err_ == cudaSuccess && dev >= 0 && dev != saved_) {
      err_ = cudaSetDevice(dev);
      switched_ = err_ == cudaSuccess;
    }
  }
  ~ScopedDevice() {
    if (switched_) cudaSetDevice(saved_);
  }
  ScopedDevice(const ScopedDevice&) = delete;
  ScopedDevice& operator=(const ScopedDevice&) = delete;
  cudaError_t error() const { return err_; }

 private:
  int saved_ = -1;
  cudaError_t err_;
  bool switched_ = false;
};

// A CUDA error as this library's status: 0, or minus the error code.
constexpr int status_of(cudaError_t e) { return e == cudaSuccess ? 0 : -static_cast<int>(e); }

int sm_count(int device);

// Error word of the kernels' bounded waits: one host-mapped, device-visible
// word per process, allocated (pinned host memory, 64 bytes) by the first
// call that launches a waiting kernel; null if that allocation failed.
unsigned int* wait_error_word();
// FA_E_TIMEOUT (and the word cleared) if a wait has given up since the last
// call, else FA_OK.  Never allocates.
int take_wait_error();

// Host-side request for the squared-difference outputs of the fused SSIM
// forward (SSIM + MSE/PSNR from one read of the frame pair).
struct SqOut {
  double psnr_bias;
  double* mse_per_image;
  double* mse_total;
  double* psnr_per_image;
  double* psnr_total;
  unsigned long long* ssd_per_image;  // uint8 input only
};

// Host-side request for GMSD from the SSIM forward's staged rows.
struct GmOut {
  double T, eps;             // GMSD threshold and epsilon in the metric's units
  double* gms_per_image;     // [N] mean of q over the image's planes
  double* gmsd_per_image;    // [N] population std of q
};

}  // namespace fab

#define FAB_TRY(EXPR)                                         \
  do {                                                        \
    if (const int st_ = ::fab::status_of(EXPR)) return st_;   \
  } while (0)

#define FAB_LAUNCH_CHECK() FAB_TRY(cudaGetLastError())

// First statement of every compute entry point: report a wait that gave up.
#define FAB_PENDING()                                          \
  do {                                                         \
    if (const int pend_ = ::fab::take_wait_error()) return pend_; \
  } while (0)

#define FAB_DEVICE_SCOPE(DEV)                                            \
  const ::fab::ScopedDevice scoped_dev_(DEV);                            \
  if (const int st_ = ::fab::status_of(scoped_dev_.error())) return st_

// bytes reserved at the head of every workspace for completion counters
#define FAB_COUNTER_BYTES 256
