// Backward selective-scan kernels, bfloat16 activations, N in {4, 8}.
#define SSM_BWD_INSTANTIATE
#include "ssm_bwd_inst.cuh"

namespace ssm {
template cudaError_t launch_bwd_n<__nv_bfloat16, 4, 4>(int, const BwdParams&, dim3, cudaStream_t);
template cudaError_t launch_bwd_n<__nv_bfloat16, 8, 4>(int, const BwdParams&, dim3, cudaStream_t);
template cudaError_t launch_bwd_n<__nv_bfloat16, 8, 2>(int, const BwdParams&, dim3, cudaStream_t);
}  // namespace ssm
