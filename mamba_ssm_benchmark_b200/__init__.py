"""B200-native (sm_100a) fused selective scan (Mamba S6): forward, backward, decode step.

Public API (reference interface it replaces in parentheses):
    selective_scan           (models/scan.py:277-299, fused-GPU scan names)
    selective_scan_triton    (kernels/triton_scan.py:322-329)
    selective_scan_fused     (scan + the mixer's D-skip and SiLU(z) gate, models/mamba.py:124)
    selective_state_update   (inline decode step, models/mamba.py:113-118)
    causal_conv1d            (the mixer's depthwise conv + SiLU, models/mamba.py:100-107)
The kernels live in libssm_b200.so (C ABI: include/ssm_b200.h); this package only marshals
torch tensors into it.  Build it with ``python -m mamba_ssm_benchmark_b200.build``.
"""

from .conv import causal_conv1d
from .decode import selective_state_update
from .scan import (SCAN_NAMES, SUPPORTED_N, SelectiveScanFn, selective_scan, selective_scan_fused,
                   selective_scan_triton)

__all__ = ["selective_scan", "selective_scan_triton", "selective_scan_fused", "selective_state_update",
           "causal_conv1d", "SelectiveScanFn", "SCAN_NAMES", "SUPPORTED_N"]
__version__ = "0.1.0"
