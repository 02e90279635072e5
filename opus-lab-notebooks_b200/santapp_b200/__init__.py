"""santapp_b200: SANTA++ sparse hierarchical sampled attention on B200 (sm_100a).

The package mirrors the hot-path entry points of the reference package
``santapp_ruler.attention`` and runs them through libsanta_b200.so, a C ABI
over hand-written CUDA kernels (see include/santa_b200.h).
"""

__version__ = "0.1.0"

from . import _lib  # noqa: F401
