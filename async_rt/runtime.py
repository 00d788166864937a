"""Reference import path for the runtime half of harp_b200.runtime.async_compat."""
from harp_b200.runtime.async_compat import (RUNTIME, AsyncModeEnd, AsyncModeStart, AsyncRunMode,  # noqa: F401
                                            AsyncSync, StreamRuntime)
