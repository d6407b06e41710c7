"""The head-sharding exchange through the library's C ABI (hx_group_*), on GPUs.

One GPU: a one-rank group gathers in place and reassembles; a rank that never
joins makes initialisation give up at its deadline with HX_ERR_NCCL instead
of hanging (host-side failure: no kernel waits on the absent peer).

Two GPUs (skipped on boxes with fewer): rank r of 2 runs the tcgen05 forward
and the backward (RoPE fused) on heads [r*H/2, (r+1)*H/2) of a B1 H8 S1024
D128 causal bf16 problem, writes its output into its slot of the group's
gather buffer, and hx_allgather_heads (NCCL all-gather + reassembly) builds
the merged [B, S, H, D] output on every rank, overlapped with the backward.
O, dK and dV must equal a single-GPU run over all heads bit for bit (heads are
independent, and each head's kernels run the same instructions in the same
order on either GPU). dQ is summed over key tiles by reduce-adds in L2 whose
order varies from run to run, so it is compared to within two bf16 spacings.
The same exchange is checked with both ranks in one process (one host thread
per GPU), and a rank that stalls between steps (alive, but never joining the
next gather) makes the other rank's gather end with HX_ERR_NCCL at its
deadline; the stalled rank then aborts its own communicator and exits (NVLS
off, plain peer copies; no rank exits while a peer's kernel may still use
its memory).
"""
import os
import threading
import time

import pytest
import torch
import torch.multiprocessing as mp

from haelixe_b200 import _native as N

pytestmark = pytest.mark.gpu

B, H, S, D = 1, 8, 1024, 128
BASE = 10000.0


def _inputs(device):
    g = torch.Generator(device="cpu").manual_seed(77)
    return [torch.randn(B, H, S, D, generator=g).to(torch.bfloat16).to(device) for _ in range(4)]


def _run(q, k, v, do, hx, o_out=None, between=None):
    scale = D ** -0.5
    qr, kr = hx.rope_forward(q, BASE), hx.rope_forward(k, BASE)
    o, lse = hx.attn_forward(qr, kr, v, scale, True, out=o_out)
    if between is not None:
        between(o)
    dq, dk, dv = hx.attn_backward(qr, kr, v, o, lse, do, scale, True, rope_base=BASE)
    return o, dq, dk, dv


def _reference():
    import haelixe_b200 as hx
    q, k, v, do = _inputs(torch.device("cuda", 0))
    o, dq, dk, dv = _run(q, k, v, do, hx)
    torch.cuda.synchronize()
    return o.permute(0, 2, 1, 3).contiguous().cpu(), dq.cpu(), dk.cpu(), dv.cpu()


def _compare(got, ref):
    ref_merged, dq, dk, dv = ref
    assert torch.equal(got["merged"], ref_merged)
    h0, h1 = got["h0"], got["h1"]
    for name, r in (("dk", dk), ("dv", dv)):
        assert torch.equal(got[name], r[:, h0:h1]), name
    a, b = got["dq"].float(), dq[:, h0:h1].float()
    spacing = torch.exp2(torch.floor(torch.log2(b.abs().clamp_min(1e-30))) - 7)
    assert ((a - b).abs() <= 2 * spacing.clamp_min(1e-6)).all()


def _rank_step(group, member, rank, world, device):
    """One sharded step on `device`: forward into the gather slot, exchange
    beside the backward, then the stream waits for the merged output."""
    import haelixe_b200 as hx
    from haelixe_b200.sharding import head_range

    torch.cuda.set_device(device)
    dev = torch.device("cuda", device)
    q, k, v, do = _inputs(dev)
    h0, h1 = head_range(rank, world, H)
    shard = [t[:, h0:h1].contiguous() for t in (q, k, v, do)]
    gbuf = group.gather_buffer((B, h1 - h0, S, D), torch.bfloat16, member)
    merged = torch.empty(B, S, H, D, device=dev, dtype=torch.bfloat16)
    o, dq, dk, dv = _run(*shard, hx, o_out=gbuf[rank],
                         between=lambda o: group.all_gather(o, merged, "bshd", member))
    group.wait(member)
    torch.cuda.synchronize(dev)
    group.sync(member)
    return {"merged": merged.cpu(), "dq": dq.cpu(), "dk": dk.cpu(), "dv": dv.cpu(), "h0": h0, "h1": h1}


def test_one_rank_group_gathers_in_place():
    from haelixe_b200.sharding import HeadGroup
    g = HeadGroup.create_rank(0, 1, 0, HeadGroup.unique_id(), timeout_ms=30000)
    try:
        assert g.info()["nranks"] == 1 and g.info()["nccl_version"] >= 22700
        got = _rank_step(g, 0, 0, 1, 0)
        _compare(got, _reference())
    finally:
        g.close()


def test_one_rank_group_merges_projection_rows_with_copies():
    """Shards stored [B, S, H, D] (heads as strided views of projection rows):
    the merge runs as copy-engine 2D copies (layout 2) and gives the same
    [B, S, H, D] output as the reassembly kernel."""
    import haelixe_b200 as hx
    from haelixe_b200.sharding import HeadGroup
    g = HeadGroup.create_rank(0, 1, 0, HeadGroup.unique_id(), timeout_ms=30000)
    try:
        q, k, v, do = _inputs(torch.device("cuda", 0))
        rows = [t.permute(0, 2, 1, 3).contiguous().permute(0, 2, 1, 3) for t in (q, k, v, do)]
        gbuf = g.gather_buffer((B, H, S, D), torch.bfloat16)
        o_slot = gbuf[0].view(B, S, H, D).permute(0, 2, 1, 3)
        merged = torch.empty(B, S, H, D, device="cuda", dtype=torch.bfloat16)
        o, dq, dk, dv = _run(*rows, hx, o_out=o_slot, between=lambda o: g.all_gather(o, merged, "bshd"))
        g.wait()
        torch.cuda.synchronize()
        g.sync()
        ref_merged, _, rdk, rdv = _reference()
        assert torch.equal(merged.cpu(), ref_merged)
        assert torch.equal(dk.cpu(), rdk) and torch.equal(dv.cpu(), rdv)
    finally:
        g.close()


def _never_joined(q):
    from haelixe_b200.sharding import HeadGroup
    torch.cuda.set_device(0)
    t0 = time.time()
    try:
        HeadGroup.create_rank(0, 2, 0, HeadGroup.unique_id(), timeout_ms=2000)
        q.put(("created", 0.0, ""))
    except N.HxError as e:
        q.put((e.status, time.time() - t0, str(e)))


def test_rank_that_never_joins_times_out():
    """Rank 0 of 2 alone: initialisation gives up after 2 s (child process, so a
    bootstrap thread left behind cannot hold this one)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_never_joined, args=(q,))
    p.start()
    status, waited, msg = q.get(timeout=120)
    p.join(timeout=60)
    if p.is_alive():
        p.kill()
    assert status == N.HX_ERR_NCCL, (status, msg)
    assert 1.5 < waited < 60, waited
    assert "aborted" in msg


def _mp_worker(rank, world, uid, out_dir, leave_after_first):
    from haelixe_b200.sharding import HeadGroup

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    g = HeadGroup.create_rank(rank, world, rank, uid, timeout_ms=20000)
    got = _rank_step(g, 0, rank, world, rank)
    torch.save(got, os.path.join(out_dir, f"rank{rank}.pt"))
    if leave_after_first:
        torch.cuda.synchronize()
        flag = os.path.join(out_dir, "leave.txt")
        if rank == 1:
            # stalls between steps (nothing of its own in flight) until rank 0
            # has given up on it, then leaves
            t0 = time.time()
            while not os.path.exists(flag) and time.time() - t0 < 120:
                time.sleep(0.05)
            g.abort()
            g.close()
            return
        # rank 0's next gather has no partner: it must end at the deadline
        g.set_timeout(3000)
        dev = torch.device("cuda", 0)
        shard = torch.zeros(B, H // world, S, D, device=dev, dtype=torch.bfloat16)
        t0 = time.time()
        status = N.HX_OK
        try:
            g.all_gather(shard, None)
            g.sync()
        except N.HxError as e:
            status = e.status
        with open(flag + ".tmp", "w") as f:
            f.write(f"{status} {time.time() - t0:.2f} {g.last_error()}")
        os.replace(flag + ".tmp", flag)
    g.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_head_sharding_matches_one_gpu(tmp_path):
    from haelixe_b200.sharding import HeadGroup
    world = 2
    mp.start_processes(_mp_worker, args=(world, HeadGroup.unique_id(), str(tmp_path), False), nprocs=world,
                       join=True, start_method="spawn")
    ref = _reference()
    for r in range(world):
        _compare(torch.load(os.path.join(tmp_path, f"rank{r}.pt")), ref)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpus_in_one_process_one_thread_each():
    from haelixe_b200.sharding import HeadGroup
    world = 2
    g = HeadGroup.create([0, 1], timeout_ms=20000)
    results, errors = {}, []

    def run(r):
        try:
            results[r] = _rank_step(g, r, r, world, r)
        except Exception as e:  # noqa: BLE001 - reported below
            errors.append(e)

    try:
        ts = [threading.Thread(target=run, args=(r,)) for r in range(world)]
        for t in ts:
            t.start()
        for t in ts:
            t.join(timeout=120)
        assert not errors, errors
        ref = _reference()
        for r in range(world):
            _compare(results[r], ref)
    finally:
        g.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_stalled_rank_ends_the_next_gather_at_its_deadline(tmp_path):
    from haelixe_b200.sharding import HeadGroup
    world = 2
    ctx = mp.get_context("spawn")
    uid = HeadGroup.unique_id()
    procs = [ctx.Process(target=_mp_worker, args=(r, world, uid, str(tmp_path), True)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
        if p.is_alive():
            p.kill()
    status, waited, *msg = open(os.path.join(tmp_path, "leave.txt")).read().split(" ")
    assert int(status) == N.HX_ERR_NCCL, (status, msg)
    assert float(waited) < 60
