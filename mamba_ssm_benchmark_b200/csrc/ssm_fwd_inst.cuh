// ssm_fwd_inst.cuh — instantiates and dispatches the forward kernels for one element type
// (SSM_ELEM, set by the including translation unit).
#pragma once
#include "ssm_fwd.cuh"

namespace ssm {

template <typename T, int N, int G, int METHOD, int MODE>
static cudaError_t launch_fwd_nm(const FwdParams& p, dim3 grid, cudaStream_t stream) {
  auto kern = ssm_fwd_kernel<N, G, METHOD, T, MODE>;
  constexpr int smem = FwdSmem<N, G, T>::BYTES;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
  }
  // one warp per CTA; grid.x counts CPW-channel slices
  dim3 g2(grid);
  g2.x = (unsigned)((p.D + Geo<N, G>::CPW - 1) / Geo<N, G>::CPW);
  kern<<<g2, 32, smem, stream>>>(p);
  return cudaGetLastError();
}

template <typename T, int N, int G>
static cudaError_t launch_fwd_n(int method, int mode, const FwdParams& p, dim3 grid, cudaStream_t stream) {
  if (mode == kModeMain) {
    switch (method) {
      case kZOH: return launch_fwd_nm<T, N, G, kZOH, kModeMain>(p, grid, stream);
      case kEuler: return launch_fwd_nm<T, N, G, kEuler, kModeMain>(p, grid, stream);
      case kBilinear: return launch_fwd_nm<T, N, G, kBilinear, kModeMain>(p, grid, stream);
    }
  } else if (mode == kModeSummary) {
    switch (method) {
      case kZOH: return launch_fwd_nm<T, N, G, kZOH, kModeSummary>(p, grid, stream);
      case kEuler: return launch_fwd_nm<T, N, G, kEuler, kModeSummary>(p, grid, stream);
      case kBilinear: return launch_fwd_nm<T, N, G, kBilinear, kModeSummary>(p, grid, stream);
    }
  } else if (mode == kModeAdjoint) {
    switch (method) {
      case kZOH: return launch_fwd_nm<T, N, G, kZOH, kModeAdjoint>(p, grid, stream);
      case kEuler: return launch_fwd_nm<T, N, G, kEuler, kModeAdjoint>(p, grid, stream);
      case kBilinear: return launch_fwd_nm<T, N, G, kBilinear, kModeAdjoint>(p, grid, stream);
    }
  }
  return cudaErrorInvalidValue;
}

// G = 2 (twice the threads for small grids) is built for N = 8 and 16.
template <>
cudaError_t launch_fwd<SSM_ELEM>(int N, int G, int method, int mode, const FwdParams& p, dim3 grid,
                                 cudaStream_t stream) {
  if (G == 2) {
    switch (N) {
      case 8: return launch_fwd_n<SSM_ELEM, 8, 2>(method, mode, p, grid, stream);
      case 16: return launch_fwd_n<SSM_ELEM, 16, 2>(method, mode, p, grid, stream);
    }
    return cudaErrorInvalidValue;
  }
  switch (N) {
    case 4: return launch_fwd_n<SSM_ELEM, 4, 4>(method, mode, p, grid, stream);
    case 8: return launch_fwd_n<SSM_ELEM, 8, 4>(method, mode, p, grid, stream);
    case 16: return launch_fwd_n<SSM_ELEM, 16, 4>(method, mode, p, grid, stream);
    case 32: return launch_fwd_n<SSM_ELEM, 32, 4>(method, mode, p, grid, stream);
    case 64: return launch_fwd_n<SSM_ELEM, 64, 4>(method, mode, p, grid, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace ssm
