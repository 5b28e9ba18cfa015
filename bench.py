#!/usr/bin/env python
"""Flagship benchmark: GPT-6.7B training step, tensor-parallel over N GPUs of one node.

    python bench.py --gpus N --steps K --warmup W            (N=1)
    torchrun --nproc-per-node N ... bench.py --gpus N ...     (N>1, one rank per GPU)

Config: 32 layers, d_model 4096, 32 heads, FFN 16384, vocab 50304,
seq 2048, micro-batch 4 (8192 tokens/step), BF16, AdamW lr 1e-4 with FP32 masters,
random-init weights, synthetic token ids; sequence-parallel fused AG->GEMM and
GEMM->RS on every linear (TP = N).  The device-timed value brackets exactly K full
optimizer steps with a barrier + synchronize on both sides and CUDA events on the
launching stream, max over ranks.  Inputs are larger than L2 (13 GB of weights per
GPU at N=1), so no flush is needed.  The end-to-end number times K calls of the
public `Trainer.train_step` with the per-step H2D copy of the token ids from pinned
host memory and the D2H read of (loss, grad norm).  Prints one JSON line on rank 0.
`--impl reference` runs the reference arm (it cannot run here: see its message).
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

BASELINE_METRIC = "GPT-6.7B TP8 train step ms (max over ranks) at 1/2/4/8 GPU; GemmRS op µs"
# Closest published full-step number of the reference lineage (8xRTX 5090, Flux BF16
# GemmOnly + NCCL reduce-scatter, same model and 8192 tokens/step).
BASELINE_MS = 984.779

REFERENCE_UNAVAILABLE = (
    "reference cannot be installed or run on B200: its source tree has no setup.py/pyproject.toml "
    "(pip: 'not installable'); its worker and codec hard-gate on RTX 5090 (compute capability 12.0, "
    "170 SMs, name check: python/flux_5090/worker.py:368, codec.py:156) and its native GEMM build needs "
    "CUTLASS 3.9.0 headers fetched over the network against third_party/cutlass.lock.json")


def parse():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--arm", default="flux")
    ap.add_argument("--transport", default="nvlink", choices=("nvlink", "nccl", "nccl_plain"),
                    help="nvlink: fused operators (product); nccl: the reference's per-block sparse all_to_all; "
                         "nccl_plain: our GEMMs with plain NCCL all_gather / reduce_scatter (unfused control)")
    ap.add_argument("--config", default="bench", choices=("bench", "small"))
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--layers", type=int, default=0, help="override the layer count (profiling only)")
    return ap.parse_args()


class ClockSampler:
    """nvidia-smi sampled every 200 ms during the timed region (rank 0)."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, enabled):
        self.enabled = enabled
        self.proc = None
        self.path = None

    def start(self):
        if not self.enabled:
            return
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append(dict(sm=float(parts[1]), max=float(parts[2]), power=float(parts[3]),
                                 hw=parts[5], hwt=parts[6], swt=parts[7], swp=parts[8]))
            except ValueError:
                continue
        os.unlink(self.path)
        if not rows:
            return None
        loaded = [r for r in rows if r["power"] > 250] or rows
        reasons = set()
        for r in rows:
            for key, name in (("hw", "hw_slowdown"), ("hwt", "hw_thermal_slowdown"),
                              ("swt", "sw_thermal_slowdown"), ("swp", "sw_power_cap")):
                if r[key].lower().startswith("active"):
                    reasons.add(name)
        return dict(sm_mhz=statistics.median(r["sm"] for r in loaded), sm_max_mhz=max(r["max"] for r in rows),
                    reasons=sorted(reasons), samples=len(rows), samples_under_load=len(loaded))


def main():
    args = parse()
    if args.impl == "reference":
        if int(os.environ.get("RANK", "0")) == 0:  # one line per job, from rank 0
            print(json.dumps({"impl": "reference", "unavailable": REFERENCE_UNAVAILABLE}))
        return 0
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from tempname_5090_b200 import config as C
    from tempname_5090_b200._native import launches
    from tempname_5090_b200.models.gpt import GPT
    from tempname_5090_b200.models.train import Trainer

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch N>1 with torchrun")
    if args.warmup < 3:
        raise SystemExit("at least 3 warm-up steps are required")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    cfg = dict(C.GPT_6P7B_BENCH if args.config == "bench" else C.SMALL)
    if args.config == "small":
        cfg.update(hidden=512, heads=4, ffn=2048, sequence=512, micro_batch=4, vocab=4096)
    if args.layers:
        cfg["layers"] = args.layers
    check = None
    if world > 1 and args.transport == "nvlink":
        # Untimed, before the model exists: the fused operators at this model's
        # layer shapes, bitwise against NCCL collectives + the same GEMM.
        from tempname_5090_b200.runner.validation import fused_operator_check
        M0 = cfg["sequence"] * cfg["micro_batch"]
        check = fused_operator_check(M0, cfg["hidden"], cfg["ffn"])
        torch.cuda.synchronize()
        if not (check["ag_bitwise_all_ranks"] and check["rs_bitwise_all_ranks"]):
            raise SystemExit(f"fused operator check failed: {check}")
    model = GPT(cfg, arm=args.arm, device=dev, transport=args.transport)
    trainer = Trainer(model)
    c = model.config
    M = c["sequence"] * c["micro_batch"]
    gen = torch.Generator().manual_seed(4321)
    host = []
    for _ in range(c["accumulation_steps"]):
        stream = torch.randint(0, c["vocab"], (c["micro_batch"], c["sequence"] + 1), generator=gen)
        host.append((stream[:, :-1].reshape(-1).contiguous().pin_memory(),
                     stream[:, 1:].reshape(-1).contiguous().pin_memory()))
    batches = [(t.to(dev), l.to(dev)) for t, l in host]

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        trainer.step(batches)
    torch.cuda.synchronize()
    warm_loss, warm_norm = trainer.step_host(batches)
    sampler = ClockSampler(rank == 0)
    sampler.start()
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = launches()
    start.record()
    for _ in range(args.steps):
        trainer.step(batches)
    end.record()
    torch.cuda.synchronize()
    barrier()
    launched = launches() - launches0
    ms = max_over_ranks(start.elapsed_time(end) / args.steps)
    e2e_ms = None
    if not args.no_e2e:
        barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            loss, norm = trainer.train_step(host)
        e2e_ms = max_over_ranks((time.perf_counter() - t0) * 1000.0 / args.steps)
    clocks = sampler.stop()
    tokens = M * c["accumulation_steps"]
    if rank == 0:
        flops = C.train_flops_per_step(c)
        line = {
            "metric": BASELINE_METRIC,
            "value": round(ms, 3),
            "unit": "ms/step",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms, 3),
            "higher_is_better": False,
            "scaling": "strong",
            "vs_baseline": round(ms / BASELINE_MS, 4),
            "baseline_ref": "984.779 ms/step: Flux BF16 GemmOnly + NCCL RS, 8xRTX 5090 (published, reference lineage)",
            "dtype": "bf16",
            "data": "synthetic token ids uniform in [0, vocab), random-init weights N(0, 0.02)",
            "impl": "ours",
            "tokens_per_s": round(tokens / (ms / 1000.0), 1),
            "model_tflops_per_gpu": round(flops / (ms / 1000.0) / world / 1e12, 1),
            "config": {"model": ("GPT-6.7B" if args.config == "bench" else "GPT-small")
                       + (f" ({c['layers']} layers: profiling, not the benchmark)" if args.layers else ""),
                       "layers": c["layers"], "hidden": c["hidden"], "heads": c["heads"], "ffn": c["ffn"],
                       "vocab": c["vocab"], "global_batch": c["micro_batch"] * c["accumulation_steps"],
                       "seq_len": c["sequence"], "tokens_per_step": tokens, "parallelism": f"tp{world}-sp",
                       "arm": args.arm, "transport": args.transport, "optimizer": "AdamW fp32 master lr 1e-4",
                       "l2": "inputs larger than L2 (weights alone exceed 126 MB)"},
            "gpu_launches": int(launched),
            "check": check,
            "warmup_loss": round(warm_loss, 4),
        }
        if e2e_ms is not None:
            line["e2e"] = {"value": round(e2e_ms, 3), "unit": "ms/step",
                           "h2d_bytes_per_step": sum(t.numel() * t.element_size() + l.numel() * l.element_size()
                                                     for t, l in host),
                           "d2h_bytes_per_step": 16,
                           "api": "Trainer.train_step(host_batches)"}
        if clocks is not None:
            line["clocks"] = clocks
        print(json.dumps(line), flush=True)
    model.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
