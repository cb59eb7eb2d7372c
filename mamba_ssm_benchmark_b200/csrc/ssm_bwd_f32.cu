// Backward selective-scan dispatch and finalize, float32 activations (kernels: ssm_bwd_f32_n*.cu).
#define SSM_ELEM float
#include "ssm_bwd_inst.cuh"
