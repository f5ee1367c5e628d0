"""TurboQuant KV cache (packed GPU storage + fused CUDA kernels)."""
from .kv_cache import (BaseKVCache, FastLloydMaxCodebook, StaticKVCache,  # noqa: F401
                       TurboQuantKVCache, _generate_rotation_matrix, build_kv_cache)
from .lloyd_max import LloydMaxCodebook, solve_lloyd_max  # noqa: F401
