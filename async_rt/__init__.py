"""Top-level `async_rt` package with the reference's import paths
(`from async_rt import is_asyncrt_enabled`, `from async_rt.runtime import
AsyncSync`, `from async_rt.async_ops import MySiLU`, ...); the implementation is
harp_b200.runtime.async_compat, on CUDA streams."""
from harp_b200.runtime.async_compat import RUNTIME, AsyncRunMode, is_asyncrt_enabled  # noqa: F401

from . import async_ops  # noqa: F401
