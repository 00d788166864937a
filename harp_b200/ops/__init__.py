"""Op layer: functional kernel wrappers and autograd modules."""
from . import functional  # noqa: F401
