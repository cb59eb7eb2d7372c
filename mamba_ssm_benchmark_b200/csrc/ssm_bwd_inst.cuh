// ssm_bwd_inst.cuh — backward kernel instantiation and dispatch for one element type.
//
// As for the forward: ssm_bwd_<type>_n<...>.cu instantiate launch_bwd_n for their N (with
// SSM_BWD_INSTANTIATE defined); ssm_bwd_<type>.cu (SSM_ELEM set) holds the dispatcher and the
// finalize kernel.
#pragma once
#include "ssm_bwd.cuh"

namespace ssm {

// Launches the backward kernel of one (element type, N, G) for any method.
template <typename T, int N, int G>
cudaError_t launch_bwd_n(int method, const BwdParams& p, dim3 grid, cudaStream_t stream);

#ifdef SSM_BWD_INSTANTIATE

template <typename T, int N, int G, int METHOD>
static cudaError_t launch_bwd_nm(const BwdParams& p, dim3 grid, cudaStream_t stream) {
  auto kern = ssm_bwd_kernel<N, G, METHOD, T>;
  constexpr int smem = BwdSmem<N, G, T>::BYTES;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
  }
  return launch_pdl(kern, grid, dim3(Geo<N, G>::NT), smem, stream, p);
}

template <typename T, int N, int G>
cudaError_t launch_bwd_n(int method, const BwdParams& p, dim3 grid, cudaStream_t stream) {
  switch (method) {
    case kZOH: return launch_bwd_nm<T, N, G, kZOH>(p, grid, stream);
    case kEuler: return launch_bwd_nm<T, N, G, kEuler>(p, grid, stream);
    case kBilinear: return launch_bwd_nm<T, N, G, kBilinear>(p, grid, stream);
  }
  return cudaErrorInvalidValue;
}

#else

// G = 2 (twice the threads for small grids) is built for N = 8 and 16.
template <>
cudaError_t launch_bwd<SSM_ELEM>(int N, int G, int method, const BwdParams& p, dim3 grid, cudaStream_t stream) {
  if (G == 2) {
    switch (N) {
      case 8: return launch_bwd_n<SSM_ELEM, 8, 2>(method, p, grid, stream);
      case 16: return launch_bwd_n<SSM_ELEM, 16, 2>(method, p, grid, stream);
    }
    return cudaErrorInvalidValue;
  }
  switch (N) {
    case 4: return launch_bwd_n<SSM_ELEM, 4, 4>(method, p, grid, stream);
    case 8: return launch_bwd_n<SSM_ELEM, 8, 4>(method, p, grid, stream);
    case 16: return launch_bwd_n<SSM_ELEM, 16, 4>(method, p, grid, stream);
    case 32: return launch_bwd_n<SSM_ELEM, 32, 4>(method, p, grid, stream);
    case 64: return launch_bwd_n<SSM_ELEM, 64, 4>(method, p, grid, stream);
  }
  return cudaErrorInvalidValue;
}

template <>
cudaError_t launch_bwd_finalize<SSM_ELEM>(const FinParams& p, cudaStream_t stream) {
  // 8 warps per block, one (b, t) row per warp for dB | dC (grid-stride beyond 16 blocks per SM)
  const long long rows = (long long)p.B * p.L;
  long long blocks = (rows + 7) / 8;
  const long long rest = ((long long)p.D * p.N + 2LL * p.D + 255) / 256;
  if (blocks < rest) blocks = rest;
  if (blocks > 148 * 16) blocks = 148 * 16;
  return launch_pdl(ssm_bwd_finalize<SSM_ELEM>, dim3((unsigned)blocks), dim3(256), 0, stream, p);
}

#endif  // SSM_BWD_INSTANTIATE

}  // namespace ssm
