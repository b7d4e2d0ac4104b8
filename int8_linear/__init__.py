"""W8A8 int8 linear layers for B200 (sm_100a): a drop-in for the int8_linear package.

The public names are those of the reference package (AshrithaG/int8-linear):
w8a8_mm, Config, NotSupported, default_config, tuned_config, plus the modules
fused_quant, vllm_patch, vllm_fuse_patch and shapes.  The kernels are hand-written
sm_100a CUDA reached through the C ABI in include/int8_linear_b200.h.

set_pdl(True) (or INT8_LINEAR_PDL=1) launches kernels with programmatic dependent
launch, for inference where weights are read-only: a kernel starts while the previous
one finishes and GEMMs prefetch their weight tiles meanwhile.
"""

from int8_linear._native import pdl_enabled, set_pdl
from int8_linear.kernel import Config, NotSupported, default_config, tuned_config, w8a8_mm, w8a8_mm_quant_act

__all__ = ["Config", "NotSupported", "default_config", "tuned_config", "w8a8_mm", "w8a8_mm_quant_act",
           "set_pdl", "pdl_enabled"]
