"""Head sharding on two GPUs with NCCL (skipped on boxes with fewer GPUs).

Rank r of 2 runs the tcgen05 forward and the backward (RoPE fused) on heads
[r*H/2, (r+1)*H/2) of a B1 H8 S1024 D128 causal bf16 problem, then
all_gather_heads (one NCCL all-gather + hx_reassemble_heads) builds the merged
[B, S, H, D] output on every rank. O, dK and dV must equal a single-GPU run
over all heads bit for bit (heads are independent, and each head's kernels
run the same instructions in the same order on either GPU). dQ is summed over
key tiles by reduce-adds in L2 whose order varies from run to run, so it is
compared to within two bf16 spacings.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

B, H, S, D = 1, 8, 1024, 128
BASE = 10000.0


def _inputs(device):
    g = torch.Generator(device="cpu").manual_seed(77)
    return [torch.randn(B, H, S, D, generator=g).to(torch.bfloat16).to(device) for _ in range(4)]


def _run(q, k, v, do, hx):
    scale = D ** -0.5
    qr, kr = hx.rope_forward(q, BASE), hx.rope_forward(k, BASE)
    o, lse = hx.attn_forward(qr, kr, v, scale, True)
    dq, dk, dv = hx.attn_backward(qr, kr, v, o, lse, do, scale, True, rope_base=BASE)
    return o, dq, dk, dv


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir):
    import datetime

    import haelixe_b200 as hx
    from haelixe_b200.sharding import all_gather_heads, head_range

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                           timeout=datetime.timedelta(seconds=60))
    try:
        q, k, v, do = _inputs(dev)
        h0, h1 = head_range(rank, world, H)
        shard = [t[:, h0:h1].contiguous() for t in (q, k, v, do)]
        o, dq, dk, dv = _run(*shard, hx)
        merged = all_gather_heads(o, layout="bshd")
        torch.cuda.synchronize()
        torch.save({"merged": merged.cpu(), "dq": dq.cpu(), "dk": dk.cpu(), "dv": dv.cpu(), "h0": h0, "h1": h1},
                   os.path.join(out_dir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_head_sharding_matches_one_gpu(tmp_path):
    import haelixe_b200 as hx
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    q, k, v, do = _inputs(torch.device("cuda", 0))
    o, dq, dk, dv = _run(q, k, v, do, hx)
    ref_merged = o.permute(0, 2, 1, 3).contiguous().cpu()
    for r in range(world):
        got = torch.load(os.path.join(tmp_path, f"rank{r}.pt"))
        assert torch.equal(got["merged"], ref_merged)
        h0, h1 = got["h0"], got["h1"]
        for name, ref in (("dk", dk), ("dv", dv)):
            assert torch.equal(got[name], ref[:, h0:h1].cpu()), name
        a, b = got["dq"].float(), dq[:, h0:h1].float().cpu()
        spacing = torch.exp2(torch.floor(torch.log2(b.abs().clamp_min(1e-30))) - 7)
        assert ((a - b).abs() <= 2 * spacing.clamp_min(1e-6)).all()
