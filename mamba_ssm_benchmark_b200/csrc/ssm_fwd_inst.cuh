// ssm_fwd_inst.cuh — forward kernel instantiation and dispatch for one element type.
//
// The kernels of one (element type, N, G) are instantiated by their own translation unit
// (ssm_fwd_<type>_n<N>.cu defines SSM_FWD_INSTANTIATE and instantiates launch_fwd_n), so the
// compiler builds them in parallel; ssm_fwd_<type>.cu (SSM_ELEM set) holds the dispatcher.
#pragma once
#include <type_traits>

#include "ssm_fwd.cuh"

namespace ssm {

// Launches the forward kernel of one (element type, N, G) for any method, mode and box size.
template <typename T, int N, int G>
cudaError_t launch_fwd_n(int method, int mode, int kb, const FwdParams& p, dim3 grid, cudaStream_t stream);

#ifdef SSM_FWD_INSTANTIATE

template <typename T, int N, int G, int METHOD, int MODE, int KB>
static cudaError_t launch_fwd_nm(const FwdParams& p, dim3 grid, cudaStream_t stream) {
  auto kern = ssm_fwd_kernel<N, G, METHOD, T, MODE, KB>;
  constexpr int smem = FwdSmem<N, G, T, KB>::BYTES;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
  }
  // one warp per CTA; grid.x counts CPW-channel slices
  dim3 g2(grid);
  g2.x = (unsigned)((p.D + Geo<N, G>::CPW - 1) / Geo<N, G>::CPW);
  return launch_pdl(kern, g2, dim3(32), smem, stream, p);
}

template <typename T, int N, int G, int MODE, int KB>
static cudaError_t launch_fwd_m(int method, const FwdParams& p, dim3 grid, cudaStream_t stream) {
  switch (method) {
    case kZOH: return launch_fwd_nm<T, N, G, kZOH, MODE, KB>(p, grid, stream);
    case kEuler: return launch_fwd_nm<T, N, G, kEuler, MODE, KB>(p, grid, stream);
    case kBilinear: return launch_fwd_nm<T, N, G, kBilinear, MODE, KB>(p, grid, stream);
  }
  return cudaErrorInvalidValue;
}

// The main pass exists with 2- and 4-tile boxes; the summary and adjoint passes (split sequences,
// short segments) use 2-tile boxes.
template <typename T, int N, int G>
cudaError_t launch_fwd_n(int method, int mode, int kb, const FwdParams& p, dim3 grid, cudaStream_t stream) {
  if (mode == kModeMain)
    return kb == 4 ? launch_fwd_m<T, N, G, kModeMain, 4>(method, p, grid, stream)
                   : launch_fwd_m<T, N, G, kModeMain, 2>(method, p, grid, stream);
  if (mode == kModeSummary) return launch_fwd_m<T, N, G, kModeSummary, 2>(method, p, grid, stream);
  if (mode == kModeAdjoint) return launch_fwd_m<T, N, G, kModeAdjoint, 2>(method, p, grid, stream);
  return cudaErrorInvalidValue;
}

#else

// G = 2 (twice the threads for small grids) is built for N = 8 and 16.
template <>
cudaError_t launch_fwd<SSM_ELEM>(int N, int G, int method, int mode, int kb, const FwdParams& p, dim3 grid,
                                 cudaStream_t stream) {
  if (G == 2) {
    switch (N) {
      case 8: return launch_fwd_n<SSM_ELEM, 8, 2>(method, mode, kb, p, grid, stream);
      case 16: return launch_fwd_n<SSM_ELEM, 16, 2>(method, mode, kb, p, grid, stream);
    }
    return cudaErrorInvalidValue;
  }
  switch (N) {
    case 4: return launch_fwd_n<SSM_ELEM, 4, 4>(method, mode, kb, p, grid, stream);
    case 8: return launch_fwd_n<SSM_ELEM, 8, 4>(method, mode, kb, p, grid, stream);
    case 16: return launch_fwd_n<SSM_ELEM, 16, 4>(method, mode, kb, p, grid, stream);
    case 32: return launch_fwd_n<SSM_ELEM, 32, 4>(method, mode, kb, p, grid, stream);
    case 64: return launch_fwd_n<SSM_ELEM, 64, 4>(method, mode, kb, p, grid, stream);
  }
  return cudaErrorInvalidValue;
}

// Dynamic shared memory of one forward CTA (one warp) with KB-tile boxes.
template <>
int fwd_smem_bytes<SSM_ELEM>(int N, int G, int kb) {
  auto pick = [&](auto n_const, auto g_const) {
    constexpr int NN = decltype(n_const)::value, GG = decltype(g_const)::value;
    return kb == 4 ? FwdSmem<NN, GG, SSM_ELEM, 4>::BYTES : FwdSmem<NN, GG, SSM_ELEM, 2>::BYTES;
  };
  using I4 = std::integral_constant<int, 4>;
  using I2 = std::integral_constant<int, 2>;
  if (G == 2) return N == 8 ? pick(std::integral_constant<int, 8>{}, I2{}) : pick(std::integral_constant<int, 16>{}, I2{});
  switch (N) {
    case 4: return pick(std::integral_constant<int, 4>{}, I4{});
    case 8: return pick(std::integral_constant<int, 8>{}, I4{});
    case 16: return pick(std::integral_constant<int, 16>{}, I4{});
    case 32: return pick(std::integral_constant<int, 32>{}, I4{});
    default: return pick(std::integral_constant<int, 64>{}, I4{});
  }
}

#endif  // SSM_FWD_INSTANTIATE

}  // namespace ssm
