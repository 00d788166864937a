"""Managers: the reference's managers/ API (shard, weight, grad, memory,
ring-attention wait engine) on the harp_b200 engine."""
from . import grad_manager, mem_manager, ring_attn_manager, shard_manager, weight_manager  # noqa: F401
