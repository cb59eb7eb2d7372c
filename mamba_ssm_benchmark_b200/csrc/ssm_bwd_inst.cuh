// ssm_bwd_inst.cuh — instantiates and dispatches the backward kernels for one element type
// (SSM_ELEM, set by the including translation unit).
#pragma once
#include "ssm_bwd.cuh"

namespace ssm {

template <typename T, int N, int METHOD>
static cudaError_t launch_bwd_nm(const BwdParams& p, dim3 grid, cudaStream_t stream) {
  auto kern = ssm_bwd_kernel<N, METHOD, T>;
  constexpr int smem = BwdSmem<N, T>::BYTES;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
  }
  kern<<<grid, Geo<N>::NT, smem, stream>>>(p);
  return cudaGetLastError();
}

template <typename T, int N>
static cudaError_t launch_bwd_n(int method, const BwdParams& p, dim3 grid, cudaStream_t stream) {
  switch (method) {
    case kZOH: return launch_bwd_nm<T, N, kZOH>(p, grid, stream);
    case kEuler: return launch_bwd_nm<T, N, kEuler>(p, grid, stream);
    case kBilinear: return launch_bwd_nm<T, N, kBilinear>(p, grid, stream);
  }
  return cudaErrorInvalidValue;
}

template <>
cudaError_t launch_bwd<SSM_ELEM>(int N, int method, const BwdParams& p, dim3 grid, cudaStream_t stream) {
  switch (N) {
    case 4: return launch_bwd_n<SSM_ELEM, 4>(method, p, grid, stream);
    case 8: return launch_bwd_n<SSM_ELEM, 8>(method, p, grid, stream);
    case 16: return launch_bwd_n<SSM_ELEM, 16>(method, p, grid, stream);
    case 32: return launch_bwd_n<SSM_ELEM, 32>(method, p, grid, stream);
    case 64: return launch_bwd_n<SSM_ELEM, 64>(method, p, grid, stream);
  }
  return cudaErrorInvalidValue;
}

template <>
cudaError_t launch_bwd_finalize<SSM_ELEM>(const FinParams& p, cudaStream_t stream) {
  const long long total = (long long)p.B * p.L * 2 * p.N + (long long)p.D * p.N + p.D;
  long long blocks = (total + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  ssm_bwd_finalize<SSM_ELEM><<<(unsigned)blocks, 256, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace ssm
