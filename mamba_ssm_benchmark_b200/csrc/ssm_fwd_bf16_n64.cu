// Forward selective-scan kernels, bfloat16 activations, N = 64.
#define SSM_FWD_INSTANTIATE
#include "ssm_fwd_inst.cuh"

namespace ssm {
template cudaError_t launch_fwd_n<__nv_bfloat16, 64, 4>(int, int, int, const FwdParams&, dim3, cudaStream_t);
}  // namespace ssm
