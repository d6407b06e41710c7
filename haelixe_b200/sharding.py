"""Head sharding across GPUs (one process per GPU).

Attention heads are independent in the forward and the backward, so rank r of
N owns heads [r*H/N, (r+1)*H/N) of every batch and needs no exchange to compute
them. The only collective is the one `MultiHeadAttention` needs afterwards:
every rank gathers all heads' outputs to merge them into the [B, S, H*D] layout
of src/nn/attention.rs:91-94. `all_gather_heads` does that with one NCCL
all-gather into a [N, B, H/N, S, D] staging buffer and one reassembly kernel
(hx_reassemble_heads) writing [B, S, H, D] directly.
"""
from __future__ import annotations

import ctypes

import torch

from . import _native as N
from .attention import _DTYPES, context


def head_range(rank: int, world: int, heads: int) -> tuple[int, int]:
    """Heads [start, stop) owned by `rank` of `world`."""
    if heads % world:
        raise ValueError(f"{heads} heads cannot be split evenly over {world} ranks")
    per = heads // world
    return rank * per, (rank + 1) * per


def reassemble_heads(gathered: torch.Tensor, out: torch.Tensor, n_shards: int, layout: str = "bshd"):
    """gathered: [n_shards, B, Hs, S, D] (contiguous) -> out [B,S,H,D] ('bshd') or [B,H,S,D]."""
    n, B, Hs, S, D = gathered.shape
    if n != n_shards:
        raise ValueError("shard count mismatch")
    ctx = context(gathered.device.index)
    ctx.use_stream()
    lay = {"bhsd": 0, "bshd": 1}[layout]
    N.check(N.lib().hx_reassemble_heads(ctx.handle, _DTYPES[gathered.dtype],
                                        ctypes.c_void_p(gathered.data_ptr()),
                                        ctypes.c_void_p(out.data_ptr()), n, B, Hs, S, D, lay),
            ctx.handle)
    return out


def all_gather_heads(o_shard: torch.Tensor, group=None, layout: str = "bshd",
                     staging: torch.Tensor | None = None, out: torch.Tensor | None = None):
    """All-gather per-rank O shards [B, H/N, S, D] and merge them.

    Returns [B, S, H, D] (layout 'bshd', i.e. [B, S, H*D] when flattened) or
    [B, H, S, D] ('bhsd'). Runs on the current stream.
    """
    import torch.distributed as dist

    world = dist.get_world_size(group)
    B, Hs, S, D = o_shard.shape
    if staging is None:
        staging = torch.empty((world,) + tuple(o_shard.shape), dtype=o_shard.dtype,
                              device=o_shard.device)
    dist.all_gather_into_tensor(staging.view(-1), o_shard.contiguous().view(-1), group=group)
    if out is None:
        shape = (B, S, world * Hs, D) if layout == "bshd" else (B, world * Hs, S, D)
        out = torch.empty(shape, dtype=o_shard.dtype, device=o_shard.device)
    return reassemble_heads(staging, out, world, layout)
