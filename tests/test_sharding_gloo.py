"""Head sharding across ranks, on CPU with the gloo backend (world size 2).

Each rank takes its heads (haelixe_b200.sharding.head_range), runs the oracle
attention forward and backward on them, and all-gathers the output shards; the
merged [B, S, H, D] result and the per-rank gradients must equal a
single-process run over all heads. The merge uses the same index mapping as
the reassembly kernel (hx_reassemble_heads), restated with numpy here.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from haelixe_b200.sharding import head_range
from oracle import oracle as ora

B, H, S, D = 2, 4, 24, 8
SCALE = 0.35


def _inputs():
    rng = np.random.default_rng(123)
    return [rng.standard_normal((B, H, S, D), dtype=np.float32) for _ in range(4)]


def merge_reference(gathered: np.ndarray) -> np.ndarray:
    """[N, B, Hs, S, D] -> [B, S, N*Hs, D], head h = r*Hs + hs (the kernel's mapping)."""
    n, b, hs, s, d = gathered.shape
    out = np.empty((b, s, n * hs, d), gathered.dtype)
    for r in range(n):
        for j in range(hs):
            out[:, :, r * hs + j, :] = gathered[r, :, j, :, :]
    return out


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q_, k_, v_, do_ = _inputs()
        h0, h1 = head_range(rank, world, H)
        sl = [a[:, h0:h1].reshape(B * (h1 - h0), S, D) for a in (q_, k_, v_, do_)]
        o, _ = ora.attn_fwd(*sl[:3], SCALE, True)
        dq, dk, dv = ora.attn_bwd(*sl, SCALE, True)
        o_shard = torch.from_numpy(o.reshape(B, h1 - h0, S, D).copy())
        parts = [torch.empty_like(o_shard) for _ in range(world)]
        dist.all_gather(parts, o_shard)
        merged = merge_reference(torch.stack(parts).numpy())
        q.put((rank, merged, dq.reshape(B, h1 - h0, S, D), dk.reshape(B, h1 - h0, S, D),
               dv.reshape(B, h1 - h0, S, D)))
    finally:
        dist.destroy_process_group()


def test_head_sharded_attention_matches_single_process():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        r, *vals = q.get(timeout=120)
        results[r] = vals
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    q_, k_, v_, do_ = _inputs()
    flat = [a.reshape(B * H, S, D) for a in (q_, k_, v_, do_)]
    o, _ = ora.attn_fwd(*flat[:3], SCALE, True)
    dq, dk, dv = (g.reshape(B, H, S, D) for g in ora.attn_bwd(*flat, SCALE, True))
    expect = o.reshape(B, H, S, D).transpose(0, 2, 1, 3)  # [B, S, H, D]
    for r in range(world):
        merged, rdq, rdk, rdv = results[r]
        np.testing.assert_allclose(merged, expect, atol=1e-6)
        h0, h1 = head_range(r, world, H)
        np.testing.assert_allclose(rdq, dq[:, h0:h1], atol=1e-6)
        np.testing.assert_allclose(rdk, dk[:, h0:h1], atol=1e-6)
        np.testing.assert_allclose(rdv, dv[:, h0:h1], atol=1e-6)


def test_head_range_partitions_heads():
    for world in (1, 2, 4, 8):
        got = [head_range(r, world, 32) for r in range(world)]
        assert got[0][0] == 0 and got[-1][1] == 32
        assert all(a[1] == b[0] for a, b in zip(got, got[1:]))
    with pytest.raises(ValueError):
        head_range(0, 3, 32)


def _leaving_worker(rank, world, port, q):
    """Rank 1 raises before the output all-gather; rank 0 must get an error, not hang."""
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    try:
        h0, h1 = head_range(rank, world, H)
        o_shard = torch.zeros(B, h1 - h0, S, D)
        if rank == 1:
            raise RuntimeError("rank 1 fails between steps")
        parts = [torch.empty_like(o_shard) for _ in range(world)]
        try:
            dist.all_gather(parts, o_shard)
            q.put((rank, "gathered"))
        except Exception as e:  # the peer left: the collective reports it
            q.put((rank, "error: " + type(e).__name__))
    except RuntimeError:
        q.put((rank, "raised"))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_rank_failure_surfaces_as_an_error_on_the_other_rank():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_leaving_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert got[1] == "raised"
    assert got[0].startswith("error"), got[0]
