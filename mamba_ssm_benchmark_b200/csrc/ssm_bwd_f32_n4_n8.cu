// Backward selective-scan kernels, float32 activations, N in {4, 8}.
#define SSM_BWD_INSTANTIATE
#include "ssm_bwd_inst.cuh"

namespace ssm {
template cudaError_t launch_bwd_n<float, 4, 4>(int, const BwdParams&, dim3, cudaStream_t);
template cudaError_t launch_bwd_n<float, 8, 4>(int, const BwdParams&, dim3, cudaStream_t);
template cudaError_t launch_bwd_n<float, 8, 2>(int, const BwdParams&, dim3, cudaStream_t);
}  // namespace ssm
