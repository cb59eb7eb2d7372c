// Forward selective-scan dispatch, float32 activations (kernels: ssm_fwd_f32_n*.cu).
#define SSM_ELEM float
#include "ssm_fwd_inst.cuh"
