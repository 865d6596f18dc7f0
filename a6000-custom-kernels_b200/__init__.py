"""B200 (sm_100a) MoE expert hot path: the pointer-table quantized MUL_MAT_ID
GEMV and its hot-expert cache, behind the reference's ggml_cuda_moe_cache_*
interface (see include/moe_cache_b200.h).

The package directory name contains hyphens; import it with
importlib.import_module("a6000-custom-kernels_b200") from the repository root.
"""
from ._lib import MoeError, build, lib  # noqa: F401
from . import moe_cache  # noqa: F401
from .moe_cache import *  # noqa: F401,F403
from .layer import MoELayer, Stack  # noqa: F401
