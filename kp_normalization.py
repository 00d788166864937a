"""Reference import path (`from kp_normalization import
replace_rmsNorm_with_kpRMSNorm`) for the RMSNorm on the harp kernels
(harp_b200.ops.modules)."""
from harp_b200.ops.modules import RMSNormFunction as CustomNormFunction  # noqa: F401
from harp_b200.ops.modules import kpRMSNorm, replace_rmsNorm_with_kpRMSNorm  # noqa: F401
