"""Reference import path for the op half of harp_b200.runtime.async_compat."""
from harp_b200.runtime.async_compat import (ApplyRotaryComplexFn, MyAdd, MyMul, MySiLU, MyTanh,  # noqa: F401
                                            add_fast, add_kernel, mm_backward_kernel, mm_kernel, mul_fast,
                                            mul_kernel, silu_backward_kernel, silu_kernel)
