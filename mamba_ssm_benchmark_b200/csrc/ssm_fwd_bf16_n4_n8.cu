// Forward selective-scan kernels, bfloat16 activations, N in {4, 8}.
#define SSM_FWD_INSTANTIATE
#include "ssm_fwd_inst.cuh"

namespace ssm {
template cudaError_t launch_fwd_n<__nv_bfloat16, 4, 4>(int, int, int, const FwdParams&, dim3, cudaStream_t);
template cudaError_t launch_fwd_n<__nv_bfloat16, 8, 4>(int, int, int, const FwdParams&, dim3, cudaStream_t);
template cudaError_t launch_fwd_n<__nv_bfloat16, 8, 2>(int, int, int, const FwdParams&, dim3, cudaStream_t);
}  // namespace ssm
