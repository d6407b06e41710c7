"""Head sharding across GPUs.

Attention heads are independent in the forward and the backward, so rank r of
N owns heads [r*H/N, (r+1)*H/N) of every batch and needs no exchange to compute
them. The only collective is the one `MultiHeadAttention` needs afterwards:
every rank gathers all heads' outputs to merge them into the [B, S, H*D] layout
of src/nn/attention.rs:91-94. `HeadGroup` does that through the library's own
C ABI (hx_group_* / hx_allgather_heads: an NCCL all-gather into a
[N, B, H/N, S, D] buffer the group owns, then the reassembly kernel writing
[B, S, H, D] directly), on a side stream so it overlaps the backward, with a
deadline on every wait. `all_gather_heads` is the same exchange for a caller
that already has a torch.distributed process group.
"""
from __future__ import annotations

import ctypes

import torch

from . import _native as N
from .attention import _DTYPES, context


class HeadGroup:
    """NCCL ranks for the head-sharding exchange (hx_group_* of the C ABI).

    One rank per process: every process calls `HeadGroup.create_rank(device,
    nranks, rank, uid)` with the same `uid` (from `HeadGroup.unique_id()` on one
    rank, shared by the caller, e.g. over torch.distributed: see `bootstrap`).
    All ranks in one process: `HeadGroup.create(devices)`, then drive member i
    from its own host thread. Every wait on a peer gives up after `timeout_ms`
    (the communicator is aborted and HxError(HX_ERR_NCCL) raised).
    """

    def __init__(self, handle, devices):
        self.handle = handle
        self.devices = list(devices)

    # ---- creation
    @staticmethod
    def unique_id() -> bytes:
        buf = ctypes.create_string_buffer(N.HX_GROUP_ID_BYTES)
        st = N.lib().hx_group_unique_id(buf)
        if st != N.HX_OK:
            raise N.HxError(st, "hx_group_unique_id failed (is libnccl.so.2 loadable?)")
        return buf.raw

    @classmethod
    def _made(cls, st, handle, devices):
        g = cls(handle, devices)
        if st != N.HX_OK:
            msg = g.last_error() if handle else ""
            g.close()
            raise N.HxError(st, msg or N.lib().hx_status_string(st).decode())
        return g

    @classmethod
    def create_rank(cls, device: int, nranks: int, rank: int, uid: bytes, flags: int = 0,
                    timeout_ms: int = 60000) -> "HeadGroup":
        if len(uid) != N.HX_GROUP_ID_BYTES:
            raise ValueError(f"the group id is {N.HX_GROUP_ID_BYTES} bytes")
        h = ctypes.c_void_p()
        st = N.lib().hx_group_create_rank(device, nranks, rank, ctypes.create_string_buffer(uid, len(uid)),
                                          flags, timeout_ms, ctypes.byref(h))
        return cls._made(st, h.value, [device])

    @classmethod
    def create(cls, devices, flags: int = 0, timeout_ms: int = 60000) -> "HeadGroup":
        arr = (ctypes.c_int * len(devices))(*devices)
        h = ctypes.c_void_p()
        st = N.lib().hx_group_create(len(devices), arr, flags, timeout_ms, ctypes.byref(h))
        return cls._made(st, h.value, devices)

    @classmethod
    def bootstrap(cls, device: int, flags: int = 0, timeout_ms: int = 60000, pg=None) -> "HeadGroup":
        """One rank per process over an initialised torch.distributed group
        (any backend): rank 0 makes the id and broadcasts it."""
        import torch.distributed as dist

        rank, world = dist.get_rank(pg), dist.get_world_size(pg)
        obj = [cls.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0, group=pg)
        return cls.create_rank(device, world, rank, obj[0], flags, timeout_ms)

    # ---- queries
    def info(self):
        n, m, v = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        N.check(N.lib().hx_group_info(self.handle, ctypes.byref(n), ctypes.byref(m), ctypes.byref(v)))
        return {"nranks": n.value, "members": m.value, "nccl_version": v.value}

    def last_error(self) -> str:
        buf = ctypes.create_string_buffer(512)
        N.lib().hx_group_last_error(self.handle, buf, 512)
        return buf.value.decode(errors="replace")

    def _check(self, st):
        if st != N.HX_OK:
            raise N.HxError(st, self.last_error() or N.lib().hx_status_string(st).decode())

    # ---- the exchange
    def gather_buffer(self, shard_shape, dtype, member: int = 0) -> torch.Tensor:
        """The group-owned gather buffer as a [nranks, *shard_shape] tensor
        (no copy). A shard written into this rank's row is gathered in place."""
        n = self.info()["nranks"]
        esize = torch.tensor([], dtype=dtype).element_size()
        count = 1
        for x in shard_shape:
            count *= int(x)
        base = ctypes.c_void_p()
        self._check(N.lib().hx_group_gather_buffer(self.handle, member, count * esize, ctypes.byref(base)))
        typestr = {2: "<f2", 4: "<f4"}[esize]
        iface = {"shape": (n,) + tuple(int(x) for x in shard_shape), "typestr": typestr,
                 "data": (base.value, False), "version": 3, "strides": None}
        holder = type("GatherBuffer", (), {"__cuda_array_interface__": iface})()
        t = torch.as_tensor(holder, device=torch.device("cuda", self.devices[member]))
        return t.view(dtype) if t.dtype != dtype else t

    def all_gather(self, shard: torch.Tensor, merged: torch.Tensor | None = None, layout: str = "bshd",
                   member: int = 0) -> torch.Tensor | None:
        """Enqueues the gather of `shard` [B, H/N, S, D] (+ the reassembly into
        `merged`, [B, S, H, D] for 'bshd', [B, H, S, D] for 'bhsd') after the
        work on the current stream; returns at once. A shard whose memory is
        [B, S, H/N, D] (the head-split view of projection rows) gathers into a
        'bshd' output with copy-engine copies instead of a kernel."""
        B, Hs, S, D = shard.shape
        rows = shard.permute(0, 2, 1, 3)
        if shard.is_contiguous():
            lay = {"bhsd": 0, "bshd": 1}[layout]
        elif rows.is_contiguous() and layout == "bshd":
            lay = 2
        else:
            raise ValueError("the shard must be contiguous as [B, H/N, S, D] or as [B, S, H/N, D]")
        ctx = context(shard.device.index)
        ctx.use_stream()
        self._check(N.lib().hx_allgather_heads(
            self.handle, member, ctx.handle, _DTYPES[shard.dtype], ctypes.c_void_p(shard.data_ptr()),
            ctypes.c_void_p(merged.data_ptr()) if merged is not None else None, B, Hs, S, D, lay))
        return merged

    def wait(self, member: int = 0, device: int | None = None):
        """The current stream waits (on the device) for the member's last gather."""
        ctx = context(self.devices[member] if device is None else device)
        ctx.use_stream()
        self._check(N.lib().hx_group_wait(self.handle, member, ctx.handle))

    def sync(self, member: int = 0):
        """Blocks until the member's last gather finished (or the timeout)."""
        self._check(N.lib().hx_group_sync(self.handle, member))

    def set_timeout(self, timeout_ms: int):
        self._check(N.lib().hx_group_set_timeout(self.handle, timeout_ms))

    def abort(self):
        N.lib().hx_group_abort(self.handle)

    def close(self):
        if self.handle:
            N.lib().hx_group_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


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
    [B, H, S, D] ('bhsd'). With a HeadGroup as `group` the exchange goes
    through the library (and the current stream waits for it); otherwise
    through torch.distributed on the current stream.
    """
    if isinstance(group, HeadGroup):
        B, Hs, S, D = o_shard.shape
        n = group.info()["nranks"]
        if out is None:
            shape = (B, S, n * Hs, D) if layout == "bshd" else (B, n * Hs, S, D)
            out = torch.empty(shape, dtype=o_shard.dtype, device=o_shard.device)
        group.all_gather(o_shard.contiguous(), out, layout)
        group.wait(device=o_shard.device.index)
        return out
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
