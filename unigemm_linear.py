"""Reference import path (`from unigemm_linear import kpLinear,
replace_linear_with_kplinear`) for the linear layer on the harp tcgen05 GEMM
(harp_b200.ops.modules)."""
from harp_b200.ops.modules import CustomLinearFunction, kpLinear, replace_linear_with_kplinear  # noqa: F401
