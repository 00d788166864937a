"""Host runtime: device error words, CUDA stream executor, memory pools."""
from . import errors  # noqa: F401
