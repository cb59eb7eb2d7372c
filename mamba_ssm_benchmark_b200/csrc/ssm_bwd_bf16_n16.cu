// Backward selective-scan kernels, bfloat16 activations, N = 16.
#define SSM_BWD_INSTANTIATE
#include "ssm_bwd_inst.cuh"

namespace ssm {
template cudaError_t launch_bwd_n<__nv_bfloat16, 16, 4>(int, const BwdParams&, dim3, cudaStream_t);
template cudaError_t launch_bwd_n<__nv_bfloat16, 16, 2>(int, const BwdParams&, dim3, cudaStream_t);
}  // namespace ssm
