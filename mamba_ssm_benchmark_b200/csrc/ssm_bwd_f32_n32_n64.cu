// Backward selective-scan kernels, float32 activations, N in {32, 64}.
#define SSM_BWD_INSTANTIATE
#include "ssm_bwd_inst.cuh"

namespace ssm {
template cudaError_t launch_bwd_n<float, 32, 4>(int, const BwdParams&, dim3, cudaStream_t);
template cudaError_t launch_bwd_n<float, 64, 4>(int, const BwdParams&, dim3, cudaStream_t);
}  // namespace ssm
