// Forward selective-scan dispatch, bfloat16 activations (kernels: ssm_fwd_bf16_n*.cu).
#define SSM_ELEM __nv_bfloat16
#include "ssm_fwd_inst.cuh"
