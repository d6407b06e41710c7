"""haelixe_b200: B200-native (sm_100a) fused attention for the haelixe crate.

The product is libhaelixe_cuda.so (C ABI: include/haelixe_cuda.h) with the C++
host layer over it (host/, libhaelixe_host.so: Device, Tensor,
FlashAttentionOp as the crate defines them). This package holds their build
recipe (build.py), the ctypes binding (_native.py),
a host-side mirror of haelixe's attention interface (attention.py), the
modules around it (nn.py: RMSNorm, Linear, MultiHeadAttention, FeedForward,
TransformerBlock, Embedding, cross_entropy, BlockStack) and the optimizer
(optim.py: AdamW).
"""
from .attention import (  # noqa: F401
    CudaAllocation,
    CudaContext,
    FlashAttentionOp,
    attn_backward,
    attn_forward,
    bin_size,
    context,
    flash_attention,
    rope_backward,
    rope_forward,
    rope_forward_qk,
    torch_arena_stats,
    use_arena_allocator,
)
from ._native import HxError  # noqa: F401
from . import nn, optim  # noqa: F401
