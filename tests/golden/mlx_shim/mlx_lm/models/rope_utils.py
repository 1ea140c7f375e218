"""Stand-in for ``mlx_lm.models.rope_utils.initialize_rope`` (no scaling)."""
from mlx.nn import RoPE


def initialize_rope(dims, base, traditional, scaling_config=None, max_position_embeddings=None):
    assert scaling_config is None
    return RoPE(dims, traditional=traditional, base=base, scale=1.0)
