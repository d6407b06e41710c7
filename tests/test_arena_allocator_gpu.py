"""Every tensor of a training loop stored in the library's arena.

use_arena_allocator() makes torch take all CUDA storage from hx_torch_malloc /
hx_torch_free: one GpuMemoryArena per device (power-of-two bins, 512-byte
floor, slabs parked on free and handed out again; src/gpu/arena.rs:13-145).
A few steps of a small TransformerBlock language model (attention, Linear,
RMSNorm, GELU, cross-entropy, AdamW) run in a fresh process with and without
it. The losses must agree, and after the first step the arena must serve the
loop from parked slabs: hits grow step after step while misses and live bytes
stay flat (a tensor kept alive across steps would show as growth).
Runs in child processes because torch's allocator can only be replaced before
the first CUDA allocation.
"""
import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import json, sys
sys.path.insert(0, sys.argv[1])
use_arena = sys.argv[2] == "1"
import torch
import haelixe_b200 as hx
if use_arena:
    hx.use_arena_allocator()
dev = torch.device("cuda", 0)
model = hx.nn.BlockStack(512, 256, 2, 2, device=dev, dtype=torch.bfloat16, rope_base=10000.0, causal=True,
                         init_std=0.02, seed=3)
params = model.parameters()
opt = hx.optim.AdamW(1e-3)
g = torch.Generator().manual_seed(5)
ids = torch.randint(0, 512, (2, 256), generator=g, dtype=torch.int32).to(dev)
tgt = torch.randint(0, 512, (2 * 256,), generator=g, dtype=torch.int32).to(dev)
out = {"loss": [], "stats": []}
for step in range(5):
    loss = model.loss(ids, tgt)
    loss.backward()
    opt.step([(q, q.grad) for q in params])
    for q in params:
        q.grad = None
    out["loss"].append(float(loss.item()))
    if use_arena:
        out["stats"].append(hx.torch_arena_stats(0))
torch.cuda.synchronize()
print("RESULT " + json.dumps(out))
"""


def _run(use_arena):
    r = subprocess.run([sys.executable, "-c", CHILD, ROOT, "1" if use_arena else "0"], capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    line = [ln for ln in r.stdout.splitlines() if ln.startswith("RESULT ")][-1]
    return json.loads(line[len("RESULT "):])


def test_training_loop_runs_from_the_arena():
    base = _run(False)
    arena = _run(True)
    for a, b in zip(arena["loss"], base["loss"]):
        assert abs(a - b) <= 1e-2 * abs(b), (arena["loss"], base["loss"])
    assert arena["loss"][-1] < arena["loss"][0]
    st = arena["stats"]
    print("arena stats per step:", st)
    assert st[0]["live_bytes"] > 0 and st[0]["misses"] > 0
    # after the first two steps (AdamW state is created on the first) the loop
    # is served from parked slabs: no new slabs, no growth of live bytes
    assert st[-1]["misses"] == st[2]["misses"], st
    assert st[-1]["live_bytes"] == st[2]["live_bytes"], st
    assert st[-1]["hits"] > st[2]["hits"], st
