"""Host-side checks of the head-sharding exchange's C ABI (hx_group_*), no GPU.

Argument checks must refuse before touching CUDA or NCCL, and the
one-rank-per-process bootstrap (rank 0 makes the NCCL id, every rank receives
the same bytes) is exercised over a two-rank gloo group on CPU.
"""
import ctypes
import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from haelixe_b200 import _native as N
from haelixe_b200.sharding import HeadGroup


def _out():
    return ctypes.c_void_p()


def test_create_rank_rejects_bad_arguments():
    L = N.lib()
    uid = b"\0" * N.HX_GROUP_ID_BYTES
    h = _out()
    for args in ((0, 0, 0, uid, 0, 1000),      # no ranks
                 (0, 2, 2, uid, 0, 1000),      # rank out of range
                 (0, 2, -1, uid, 0, 1000),
                 (-1, 2, 0, uid, 0, 1000),     # bad device
                 (0, 2, 0, None, 0, 1000),     # no id
                 (0, 2, 0, uid, 0, 0),         # no timeout
                 (0, 2, 0, uid, 64, 1000)):    # unknown flag
        assert L.hx_group_create_rank(*args, ctypes.byref(h)) == N.HX_ERR_INVALID, args
        assert h.value is None
    assert L.hx_group_create_rank(0, 2, 0, uid, 0, 1000, None) == N.HX_ERR_INVALID


def test_create_rejects_bad_arguments():
    L = N.lib()
    h = _out()
    devs = (ctypes.c_int * 2)(0, 0)
    assert L.hx_group_create(0, devs, 0, 1000, ctypes.byref(h)) == N.HX_ERR_INVALID
    assert L.hx_group_create(2, None, 0, 1000, ctypes.byref(h)) == N.HX_ERR_INVALID
    assert L.hx_group_create(2, devs, 0, -5, ctypes.byref(h)) == N.HX_ERR_INVALID
    assert L.hx_group_create(2, devs, 8, 1000, ctypes.byref(h)) == N.HX_ERR_INVALID


def test_calls_on_no_group_are_refused():
    L = N.lib()
    assert L.hx_group_destroy(None) == N.HX_OK
    assert L.hx_group_abort(None) == N.HX_ERR_INVALID
    assert L.hx_group_sync(None, 0) == N.HX_ERR_INVALID
    assert L.hx_group_wait(None, 0, None) == N.HX_ERR_INVALID
    assert L.hx_group_set_timeout(None, 10) == N.HX_ERR_INVALID
    assert L.hx_allgather_heads(None, 0, None, N.HX_BF16, None, None, 1, 1, 1, 64, 1) == N.HX_ERR_INVALID
    base = _out()
    assert L.hx_group_gather_buffer(None, 0, 16, ctypes.byref(base)) == N.HX_ERR_INVALID
    buf = ctypes.create_string_buffer(8)
    assert L.hx_group_last_error(None, buf, 8) == N.HX_ERR_INVALID


def test_unique_id_is_fresh_and_sized():
    a, b = HeadGroup.unique_id(), HeadGroup.unique_id()
    assert len(a) == len(b) == N.HX_GROUP_ID_BYTES
    assert a != b


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _bootstrap_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        obj = [HeadGroup.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        q.put((rank, obj[0]))
    finally:
        dist.destroy_process_group()


def test_bootstrap_id_reaches_every_rank_over_gloo():
    """The id exchange HeadGroup.bootstrap performs before creating its rank."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_bootstrap_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert len(got[0]) == N.HX_GROUP_ID_BYTES and got[0] == got[1]
