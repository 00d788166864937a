"""Reference import path (`from kp_multi_tensor_adamw import
kp_multi_tensor_adamw`) for the multi-tensor AdamW on the harp kernel
(harp_b200.ops.modules)."""
from harp_b200.ops.modules import kp_multi_tensor_adamw  # noqa: F401
