"""Model zoo: DiT (flagship), Z-Image (reference layout), MMDiT, Flux."""
from .dit import DiT, DiTConfig, PRESETS as DIT_PRESETS  # noqa: F401
