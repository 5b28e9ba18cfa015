"""torchrun worker for the multi-GPU tests (one rank per GPU, NCCL + NVLink IPC).

    torchrun --nproc-per-node W --master-addr 127.0.0.1 tests/multigpu_worker.py --case NAME

Exits 0 when every check passes on every rank; prints `CASE-OK <name>` on rank 0.
"""
import argparse
import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def require(ok, msg):
    flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device="cuda")
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    if int(flag.item()) != 1:
        raise RuntimeError(msg + " (failed on at least one rank)")


def case_gemm_rs(rank, world):
    from tempname_5090_b200.parallel.gemm_rs import GemmRS
    from tempname_5090_b200.ops import gemm as G, taco
    from tempname_5090_b200._native import check_status
    m, n, k, chunk = world * 512, 1024, 768, 128
    rows = m // world
    g = torch.Generator(device="cuda").manual_seed(100 + rank)
    x = torch.randn((m, k), generator=g, device="cuda").to(torch.bfloat16)
    w = (0.05 * torch.randn((n, k), generator=g, device="cuda")).to(torch.bfloat16)
    partial = G.matmul(x, w, bn=256)
    gathered = torch.empty_like(partial)
    dist.all_to_all_single(gathered, partial)
    sources = gathered.view(world, rows, n)
    outputs = {}
    from tempname_5090_b200.parallel import planning
    plan = planning.make_role(m, n, k, world, chunk, planning.candidates(m, n, k, world, chunk)[1]["arrival_order"])
    for arm in ("flux", "flux_taco", "flux_taco_interleaved", "flux_taco_interleaved_arrival"):
        p = plan if arm.endswith("arrival") else None
        op = GemmRS(m, n, k, arm=arm, chunk_rows=chunk, plan=p)
        for _ in range(3):
            out = op.forward(x, w)
        torch.cuda.synchronize()
        check_status()
        local = sources[rank].contiguous()
        if op.quantized:
            blocks = []
            for b in range(rows // chunk):
                pk = [taco.encode(sources[s][b * chunk:(b + 1) * chunk].contiguous()) for s in range(world) if s != rank]
                blocks.append(taco.decode_reduce(local[b * chunk:(b + 1) * chunk].contiguous(), torch.cat(pk), rank, world))
            expect = torch.cat(blocks)
        else:
            remote = torch.cat([sources[s] for s in range(world) if s != rank])
            expect = taco.ordered_reduce(local, remote, rank, world)
        require(torch.equal(out, expect), f"GemmRS {arm} differs from all_to_all + ordered reduce")
        outputs[arm] = out
        nccl = GemmRS(m, n, k, arm=arm, chunk_rows=chunk, plan=p, transport="nccl").forward(x, w)
        torch.cuda.synchronize()
        require(torch.equal(nccl, out), f"NCCL transport differs from NVLink transport for {arm}")
        op.close()
    require(torch.equal(outputs["flux_taco"], outputs["flux_taco_interleaved"]) and
            torch.equal(outputs["flux_taco"], outputs["flux_taco_interleaved_arrival"]),
            "TACO arms are not bitwise equal")


def case_scatter(rank, world):
    """TensorParallel.scatter_sum (the embedding's SumScatter) over the pull
    transport equals NCCL reduce_scatter on embedding-like inputs (one non-zero
    source per row), bitwise, back to back."""
    from tempname_5090_b200.parallel.tp import TensorParallel
    from tempname_5090_b200._native import check_status
    tp = TensorParallel(None)
    m, n = world * 512, 1024
    for it in range(3):
        g = torch.Generator(device="cuda").manual_seed(50 + it)
        owner = torch.randint(0, world, (m,), generator=g, device="cuda")
        x = torch.randn((m, n), generator=torch.Generator(device="cuda").manual_seed(60 + rank + 10 * it),
                        device="cuda").to(torch.bfloat16) * (owner == rank)[:, None].to(torch.bfloat16)
        got = tp.scatter_sum(x)
        want = torch.empty_like(got)
        dist.reduce_scatter_tensor(want, x)
        torch.cuda.synchronize()
        check_status()
        require(torch.equal(got, want), "pull scatter differs from NCCL reduce_scatter")
    tp.close()


def case_ag_gemm(rank, world):
    from tempname_5090_b200.parallel.ag_gemm import AGGemm
    from tempname_5090_b200.ops import gemm as G
    from tempname_5090_b200._native import check_status
    m, k, n = world * 256, 512, 1536
    g = torch.Generator(device="cuda").manual_seed(7 + rank)
    shard = torch.randn((m // world, k), generator=g, device="cuda").to(torch.bfloat16)
    w = (0.05 * torch.randn((n, k), generator=torch.Generator(device="cuda").manual_seed(1), device="cuda")).to(torch.bfloat16)
    full = torch.empty((m, k), dtype=torch.bfloat16, device="cuda")
    dist.all_gather_into_tensor(full, shard)
    op = AGGemm(m, k, n=n)
    kind = op.tile_kind(n, 256)
    for it in range(6):
        s = (shard * (it + 1)).to(torch.bfloat16)
        f = (full * (it + 1)).to(torch.bfloat16)
        if it % 2:  # the producer writes the shard straight into the gather buffer
            buf = op.input_buffer()
            buf.copy_(s)
            s = buf
        out = op.forward(s, w, bn=256)  # back to back: no host barrier between calls
        torch.cuda.synchronize()
        check_status()
        require(torch.equal(op.gathered, f) and torch.equal(out, G.matmul(f, w, bn=256, pair=kind)),
                "AG->GEMM mismatch")
    op.close()
    # Eight 128-row blocks per rank on 20 communication CTAs, shard copied by
    # the gatherers: a CTA copies one own block and then waits for a peer's
    # block whose owner CTA is in the same position, so own blocks must be
    # published before that wait (a lazily published own block deadlocked here).
    m2, k2, n2 = world * 1024, 256, 512
    shard2 = torch.randn((m2 // world, k2), generator=g, device="cuda").to(torch.bfloat16)
    w2 = (0.05 * torch.randn((n2, k2), generator=g, device="cuda")).to(torch.bfloat16)
    full2 = torch.empty((m2, k2), dtype=torch.bfloat16, device="cuda")
    dist.all_gather_into_tensor(full2, shard2)
    op = AGGemm(m2, k2, comm_ctas=20, n=n2)
    for _ in range(2):
        out = op.forward(shard2, w2, bn=256)
        torch.cuda.synchronize()
        check_status()
        require(torch.equal(op.gathered, full2) and
                torch.equal(out, G.matmul(full2, w2, bn=256, pair=op.tile_kind(n2, 256))),
                "AG->GEMM mismatch (copied shard, eight blocks per rank)")
    op.close()


def case_model(rank, world):
    from tempname_5090_b200.models.gpt import GPT
    from tempname_5090_b200.models.train import Trainer
    from tempname_5090_b200._native import check_status
    cfg = dict(layers=2, hidden=1024, ffn=4096, heads=8, sequence=512, micro_batch=2,
               accumulation_steps=1, vocab=4096, chunk_rows=128)
    for arm in ("flux", "flux_taco"):
        model = GPT(cfg, arm=arm, device="cuda", seed=21)
        g = torch.Generator().manual_seed(3)
        M = cfg["sequence"] * cfg["micro_batch"]
        tokens = torch.randint(0, cfg["vocab"], (M,), generator=g).cuda()
        targets = torch.randint(0, cfg["vocab"], (M,), generator=g).cuda()
        loss = model.forward_backward(tokens, targets)
        torch.cuda.synchronize()
        check_status()
        shards = [None] * world
        dist.all_gather_object(shards, {k: v.cpu() for k, v in model.state_dict().items()})
        grads = [None] * world
        dist.all_gather_object(grads, {k: model.g[k].cpu() for k in model.state_dict()})
        if rank == 0:
            sys.path.insert(0, os.path.join(ROOT, "tests"))
            from test_model_cpu import assemble_dense
            from tempname_5090_b200.config import validate_config
            dense = assemble_dense(shards, validate_config(cfg, 1), world)
            single = GPT(cfg, group="local", device="cpu", seed=0, init=False)
            single.load_state_dict(dense)
            ref = single.forward_backward(tokens.cpu(), targets.cpu())
            tol = 2e-2 if arm == "flux" else 6e-2
            ok = abs(loss.item() - ref.item()) < tol * abs(ref.item())
            dg = assemble_dense(grads, validate_config(cfg, 1), world)
            for name in ("embedding", "layers.1.fc1_weight", "layers.0.qkv_weight", "layers.0.attn_weight"):
                r = ((dg[name].float() - single.g[name].float()).norm() / single.g[name].float().norm()).item()
                ok = ok and r < 10 * tol
        else:
            ok = True
        require(ok, f"TP{world} model ({arm}) differs from the single-rank model")
        trainer = Trainer(model)
        for _ in range(3):
            lv, nv = trainer.train_step([(tokens.cpu(), targets.cpu())])
        vals = torch.tensor([lv, nv], dtype=torch.float64, device="cuda")
        lo, hi = vals.clone(), vals.clone()
        dist.all_reduce(lo, op=dist.ReduceOp.MIN)
        dist.all_reduce(hi, op=dist.ReduceOp.MAX)
        require(torch.equal(lo, hi), "ranks disagree on loss / grad norm")
        model.close()


def case_missing_peer(rank, world):
    """Rank world-1 skips one GemmRS call (learned on the host via the store);
    the others' receivers time out after 1 s with status 5 and stay usable."""
    from tempname_5090_b200.parallel.gemm_rs import GemmRS
    from tempname_5090_b200._native import status_tensor
    m, n, k = world * 256, 512, 256
    op = GemmRS(m, n, k, timeout_ns=1_000_000_000)
    x = torch.randn((m, k), device="cuda").to(torch.bfloat16)
    w = torch.randn((n, k), device="cuda").to(torch.bfloat16)
    op.forward(x, w)
    torch.cuda.synchronize()
    dist.barrier()
    status = status_tensor("cuda")
    status.zero_()
    if rank != world - 1:
        op.forward(x, w)  # peer never pushes: bounded waits expire
        torch.cuda.synchronize()
        code = int(status[0].item())
        assert code == 5, f"expected peer-flag timeout status, got {code}"
        status.zero_()
        assert torch.ones(4, device="cuda").sum().item() == 4.0  # context usable
    torch.cuda.synchronize()
    dist.barrier()


CASES = dict(gemm_rs=case_gemm_rs, ag_gemm=case_ag_gemm, model=case_model, missing_peer=case_missing_peer,
             scatter=case_scatter)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", required=True, choices=sorted(CASES))
    args = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    try:
        CASES[args.case](rank, world)
        dist.barrier()
        if rank == 0:
            print(f"CASE-OK {args.case}", flush=True)
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
