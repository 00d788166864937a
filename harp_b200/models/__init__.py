"""Model zoo: DiT (flagship), Z-Image (reference layout), MMDiT, Flux."""
from .dit import DiT, DiTConfig, PRESETS as DIT_PRESETS  # noqa: F401
from .mmdit import MMDiT, MMDiTConfig, PRESETS as MMDIT_PRESETS  # noqa: F401
from .zimage import PRESETS as ZIMAGE_PRESETS, ZImageTransformer2DModel, Z_Transformer  # noqa: F401
