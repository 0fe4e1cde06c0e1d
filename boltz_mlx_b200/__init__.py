"""B200-native pairformer triangle attention (starting + ending node, forward).

Drop-in for boltz_mlx.layers.triangular_attention.attention.TriangleAttention of
jackryan225/boltz-mlx: same constructor, parameter names and call, computed by hand-written sm_100a
CUDA kernels in libtriattn.so (C ABI: include/triattn.h).
"""

from .triangle_attention import (  # noqa: F401
    Attention,
    TriangleAttention,
    TriangleAttentionEndingNode,
    TriangleAttentionStartingNode,
    load_params,
    pack_weights,
)
from .triangle_mult import (  # noqa: F401
    TriangleMultiplicationIncoming,
    TriangleMultiplicationOutgoing,
    load_trimul_params,
)
from . import _lib  # noqa: F401
from .weights import load_module, load_pairformer_triatt, read_safetensors, write_safetensors  # noqa: F401

__all__ = ["Attention", "TriangleAttention", "TriangleAttentionStartingNode", "TriangleAttentionEndingNode",
           "load_params", "pack_weights", "read_safetensors", "write_safetensors", "load_module",
           "load_pairformer_triatt", "TriangleMultiplicationOutgoing", "TriangleMultiplicationIncoming",
           "load_trimul_params"]
