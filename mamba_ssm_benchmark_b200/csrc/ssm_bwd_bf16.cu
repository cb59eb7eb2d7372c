// Backward selective-scan dispatch and finalize, bfloat16 activations (kernels: ssm_bwd_bf16_n*.cu).
#define SSM_ELEM __nv_bfloat16
#include "ssm_bwd_inst.cuh"
