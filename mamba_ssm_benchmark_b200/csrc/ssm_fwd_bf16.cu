// Forward selective-scan kernels, bfloat16 activations (float32 state and accumulation).
#define SSM_ELEM __nv_bfloat16
#include "ssm_fwd_inst.cuh"
