// Scales a unit gradient by the upstream gradient once it is known:
//   out[i] = in[i] * (float)(s[i / per_image] * mult)      (per_image_scale)
//   out[i] = in[i] * (float)(s[0] * mult)                  (otherwise)
// The fused SSIM value+gradient launch produces the gradient of the batch
// mean for an upstream gradient of 1; this is the only pass left for the
// backward.  float4 loads and stores when every image is a multiple of 4
// floats and both buffers are 16-byte aligned, scalar otherwise.
#include "common.cuh"

namespace fab {

template <bool VEC>
__global__ void __launch_bounds__(256) grad_scale_kernel(const float* in,
                                                          long long per_image, long long total,
                                                          const double* __restrict__ s,
                                                          int per_image_scale, double mult,
                                                          float* out) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  const bool inplace = in == out;
  // in place with a single factor of exactly 1: nothing changes
  if (inplace && !per_image_scale && (float)(__ldg(s) * mult) == 1.0f) return;
  if constexpr (VEC) {
    const long long n4 = total >> 2, pi4 = per_image >> 2;
    const float4* in4 = reinterpret_cast<const float4*>(in);
    float4* out4 = reinterpret_cast<float4*>(out);
    const float f0 = (float)(__ldg(s) * mult);
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
      const float f = per_image_scale ? (float)(__ldg(s + i / pi4) * mult) : f0;
      if (inplace && f == 1.0f) continue;
      float4 v = __ldcs(in4 + i);
      v.x *= f; v.y *= f; v.z *= f; v.w *= f;
      __stcs(out4 + i, v);
    }
  } else {
    const float f0 = (float)(__ldg(s) * mult);
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
      const float f = per_image_scale ? (float)(__ldg(s + i / per_image) * mult) : f0;
      if (inplace && f == 1.0f) continue;
      out[i] = in[i] * f;
    }
  }
}

int grad_scale_impl(const float* in, long long per_image, int n, const double* s,
                    int per_image_scale, double mult, float* out, int device, cudaStream_t st) {
  if (!in || !out || !s) return FA_E_ARG;
  if (n <= 0 || per_image <= 0) return FA_E_SHAPE;
  const long long total = per_image * n;
  const bool vec = (per_image % 4 == 0) &&
                   ((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) & 15u) == 0;
  const long long work = vec ? total / 4 : total;
  long long blocks = (work + 255) / 256;
  const long long cap = (long long)sm_count(device) * 8;
  if (blocks > cap) blocks = cap;
  if (vec)
    grad_scale_kernel<true><<<(unsigned)blocks, 256, 0, st>>>(in, per_image, total, s,
                                                              per_image_scale, mult, out);
  else
    grad_scale_kernel<false><<<(unsigned)blocks, 256, 0, st>>>(in, per_image, total, s,
                                                               per_image_scale, mult, out);
  FAB_LAUNCH_CHECK();
  return FA_OK;
}

}  // namespace fab
