"""Reference import path (`from kp_rope import kp_apply_rotary_emb`): rotary
embedding of x [B, H, S, D] by complex freqs_cis, on harp's
ApplyRotaryComplexFn.  As in the reference, only the complex form exists."""
from harp_b200.ops.modules import ApplyRotaryComplexFn


def kp_apply_rotary_emb(x, freqs_cis, use_real: bool = True, use_real_unbind_dim: int = -1):
    if use_real:
        raise NotImplementedError("kp_apply_rotary_emb: only the complex form (use_real=False)")
    return ApplyRotaryComplexFn.apply(x, freqs_cis)
