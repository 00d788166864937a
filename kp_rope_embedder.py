"""Reference import path (`from kp_rope_embedder import
replace_ropeembedder_with_sverope`) for the Z-Image rotary embedders
(harp_b200.models.zimage).  RopeEmbedderReference computes the angles per
call and RopeEmbedderSVE gathers from per-device tables; both return fp32
(cos, sin) pairs [N, D/2, 2], and `.complex(ids)` gives the reference's
complex64 [N, D/2]."""
from harp_b200.models.zimage import RopeEmbedder as RopeEmbedderReference  # noqa: F401
from harp_b200.models.zimage import RopeTableEmbedder as RopeEmbedderSVE  # noqa: F401
from harp_b200.models.zimage import replace_ropeembedder_with_sverope  # noqa: F401
