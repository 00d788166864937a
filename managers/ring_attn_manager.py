"""Reference import path for harp_b200.managers.ring_attn_manager."""
from harp_b200.managers.ring_attn_manager import *  # noqa: F401,F403
from harp_b200.managers import ring_attn_manager as _impl

__all__ = [n for n in dir(_impl) if not n.startswith("_")]
globals().update({n: getattr(_impl, n) for n in __all__})
