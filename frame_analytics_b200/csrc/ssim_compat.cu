// Kernels of the reference-compatible SSIM entry points (fa_cuda_ssim,
// fa_cuda_ssim_cs, fa_cuda_ssim_backward, fa_cuda_ssim_cs_backward).  Those
// calls pass the Gaussian window as a device pointer (the reference's
// frame_analytics/csrc/fa_abi.h:139-200), so these instantiations read their
// taps from it in the kernel prologue (load_device_taps) instead of taking
// them in the launch parameters.  The host never reads the window: no copy,
// no synchronisation, and a window freed and reallocated at the same address
// is simply read again.  They stage rows with register loads, which serve any
// window, symmetric or not.
#include "ssim_bwd.cuh"
#include "ssim_fwd.cuh"

namespace fab {

template <typename T, bool CS>
static int fwd_dw_k(const SsimArgs& p, int K, int device, cudaStream_t st) {
  switch (K) {
    case 11: return launch_fwd<T, 11, CS, STAGE_GENERIC, false, true>(p, device, st);
    case 9: return launch_fwd<T, 9, CS, STAGE_GENERIC, false, true>(p, device, st);
    case 7: return launch_fwd<T, 7, CS, STAGE_GENERIC, false, true>(p, device, st);
    case 5: return launch_fwd<T, 5, CS, STAGE_GENERIC, false, true>(p, device, st);
    case 3: return launch_fwd<T, 3, CS, STAGE_GENERIC, false, true>(p, device, st);
    default: return FA_E_WINDOW;
  }
}

template <typename T>
static int fwd_dw_t(const SsimArgs& p, bool cs, int K, int device, cudaStream_t st) {
  return cs ? fwd_dw_k<T, true>(p, K, device, st) : fwd_dw_k<T, false>(p, K, device, st);
}

// The dtypes of the reference's fa_cuda_ssim (fa_abi.h:43-48).
int fwd_dw_dispatch(const SsimArgs& p, int dtype, bool cs, int K, int device, cudaStream_t st) {
  switch (dtype) {
    case FA_U8: return fwd_dw_t<unsigned char>(p, cs, K, device, st);
    case FA_F16: return fwd_dw_t<f16_t>(p, cs, K, device, st);
    case FA_BF16: return fwd_dw_t<bf16_t>(p, cs, K, device, st);
    case FA_F32: return fwd_dw_t<float>(p, cs, K, device, st);
    case FA_F64: return fwd_dw_t<double>(p, cs, K, device, st);
    default: return FA_E_DTYPE;
  }
}

template <int GMODE>
static int bwd_dw_k(const SsimArgs& p, int K, int device, cudaStream_t st) {
  switch (K) {
    case 11: return launch_bwd_general<11, true, true, GMODE, STAGE_GENERIC, false, true>(p, device, st);
    case 9: return launch_bwd_general<9, true, true, GMODE, STAGE_GENERIC, false, true>(p, device, st);
    case 7: return launch_bwd_general<7, true, true, GMODE, STAGE_GENERIC, false, true>(p, device, st);
    case 5: return launch_bwd_general<5, true, true, GMODE, STAGE_GENERIC, false, true>(p, device, st);
    case 3: return launch_bwd_general<3, true, true, GMODE, STAGE_GENERIC, false, true>(p, device, st);
    default: return FA_E_WINDOW;
  }
}

int bwd_dw_dispatch(const SsimArgs& p, int gmode, int K, int device, cudaStream_t st) {
  switch (gmode) {
    case G_MAP: return bwd_dw_k<G_MAP>(p, K, device, st);
    case G_SCALAR: return bwd_dw_k<G_SCALAR>(p, K, device, st);
    case G_PLANE: return bwd_dw_k<G_PLANE>(p, K, device, st);
    default: return FA_E_ARG;
  }
}

}  // namespace fab
