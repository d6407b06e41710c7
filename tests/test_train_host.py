"""CPU tests of the training-step host logic (no GPU): module structure and
parameter counts of FeedForward / TransformerBlock / BlockStack (nn/mlp.rs,
nn/transformer.rs), AdamW's defaults and argument checks (optim.rs:100-126),
and that every op refuses CPU tensors instead of falling back to a CPU path."""
import pytest
import torch

import haelixe_b200 as hx


def test_feed_forward_and_block_structure():
    ff = hx.nn.FeedForward(32)
    assert tuple(ff.linear1.weight.shape) == (32, 128) and tuple(ff.linear2.weight.shape) == (128, 32)
    blk = hx.nn.TransformerBlock(32, 4)
    # norm1, mha (norm + 4 linears), norm2, mlp (2 linears): the reference's field order
    shapes = [tuple(p.shape) for p in blk.parameters()]
    assert shapes == [(32,), (32,), (32, 32), (32,), (32, 32), (32,), (32, 32), (32,), (32, 32), (32,), (32,),
                      (32, 128), (128,), (128, 32), (32,)]
    assert all(p.requires_grad for p in blk.parameters())
    assert torch.equal(blk.norm1.weight, torch.ones(32))  # rms_norm.rs: weights start at 1


def test_block_stack_parameter_count_and_init():
    V, Hd, H, L = 50, 64, 4, 3
    m = hx.nn.BlockStack(V, Hd, H, L, init_std=0.02, seed=3)
    # mha: norm + 4 Linears; norm1, norm2; mlp: two Linears
    per_block = (Hd + 4 * (Hd * Hd + Hd)) + 2 * Hd + (Hd * 4 * Hd + 4 * Hd) + (4 * Hd * Hd + Hd)
    want = V * Hd + L * per_block + Hd + (Hd * V + V)
    assert sum(p.numel() for p in m.parameters()) == want
    w = m.blocks[0].mlp.linear1.weight
    assert abs(float(w.detach().std()) - 0.02) < 0.003  # N(0, 0.02) re-draw of the Linear weights
    m2 = hx.nn.BlockStack(V, Hd, H, L, init_std=0.02, seed=3)
    assert all(torch.equal(a, b) for a, b in zip(m.parameters(), m2.parameters()))  # seeded


def test_ops_refuse_cpu_tensors():
    x = torch.zeros(2, 8)
    with pytest.raises(RuntimeError, match="CUDA"):
        hx.nn.gelu(x)
    with pytest.raises(RuntimeError, match="CUDA"):
        hx.nn.cross_entropy(x, torch.zeros(2, dtype=torch.int32))
    with pytest.raises(RuntimeError, match="CUDA"):
        hx.nn.embedding(torch.zeros(3, dtype=torch.int32), x)
    with pytest.raises(RuntimeError, match="CUDA"):
        hx.nn.BlockStack(10, 16, 2, 1)(torch.zeros(1, 4, dtype=torch.int32))


def test_adamw_defaults_and_checks():
    opt = hx.optim.AdamW(1e-3)
    assert (opt.beta1, opt.beta2, opt.eps, opt.weight_decay) == (0.9, 0.999, 1e-8, 0.01)
    opt.set_lr(5e-4)
    assert opt.lr == 5e-4
    p = torch.zeros(4, requires_grad=True)
    with pytest.raises(ValueError, match="CUDA"):
        opt.step([(p, torch.zeros(4))])
    opt.step([(p, None)])  # parameters without a gradient are skipped
    opt.zero_grad()
