"""Vocab-parallel cross-entropy on two Gloo ranks against F.cross_entropy in
FP64 (forward loss and the in-place dlogits), targets on both vocabulary shards.
Follows the reference's FP64 check (tests/test_model_contract.py:108-137 of
TempName-5090)."""
import os
import socket
import tempfile

import torch
import torch.nn.functional as F

M, V = 64, 1024


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _data():
    g = torch.Generator().manual_seed(17)
    logits = (3.0 * torch.randn((M, V), generator=g)).to(torch.bfloat16)
    targets = torch.randint(0, V, (M,), generator=g)
    return logits, targets


def _worker(rank, world, port, out_dir):
    import torch.distributed as dist
    from tempname_5090_b200.ops import loss as CE
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        logits, targets = _data()
        shard = logits[:, rank * V // world:(rank + 1) * V // world].clone()
        loss, state = CE.forward(shard, targets, None, rank, world)
        CE.backward(shard, targets, state, 1.0 / M)
        torch.save(dict(loss=loss, grad=shard), os.path.join(out_dir, f"r{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_vocab_parallel_ce_matches_fp64_reference():
    import torch.multiprocessing as mp
    world = 2
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(world, _port(), d), nprocs=world, join=True)
        res = [torch.load(os.path.join(d, f"r{r}.pt")) for r in range(world)]
    logits, targets = _data()
    x = logits.double().requires_grad_(True)
    ref = F.cross_entropy(x, targets)
    ref.backward()
    for r in res:
        assert abs(r["loss"].item() - ref.item()) <= 1e-5 * abs(ref.item())
    grad = torch.cat([r["grad"] for r in res], 1).double()
    assert ((grad - x.grad).norm() / x.grad.norm()).item() < 1e-2  # BF16 output
    assert torch.equal(res[0]["loss"], res[1]["loss"])
