// Forward selective-scan kernels, float32 activations.
#define SSM_ELEM float
#include "ssm_fwd_inst.cuh"
