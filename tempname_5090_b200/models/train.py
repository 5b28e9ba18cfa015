"""Training step: micro-batch forward/backward, replicated-gradient all-reduce,
global FP64 gradient norm, on-device clipping and fused FP32-master AdamW.

Policy (TempName-5090 python/flux_5090/model.py:382-425):
* micro-batch gradients accumulate in FP32 when accumulation_steps > 1;
* replicated parameters' gradients are summed over the TP group;
* the global norm counts sharded gradients on every rank and replicated ones
  once (rank 0), in FP64, all-reduced over the TP group;
* clip coefficient min(max_norm / (norm + 1e-6), 1) applied inside AdamW;
* AdamW betas (0.9, 0.95), eps 1e-8, weight decay on >= 2-D parameters only;
* the FP32 master is copied back to the BF16 parameters.
`step()` never waits on the host; `step_host()` additionally reads the loss
and norm back (one device->host copy) and raises on a non-finite result.
"""
from __future__ import annotations

import math

import torch

from .._native import check_status
from ..ops import optim as O
from .gpt import GPT
from ..utils import tracing


class Trainer:
    def __init__(self, model: GPT, *, lr: float | None = None, weight_decay: float | None = None,
                 betas=(0.9, 0.95), eps: float = 1e-8, max_grad_norm: float | None = None):
        c = model.config
        self.model = model
        self.lr = c["learning_rate"] if lr is None else lr
        self.weight_decay = c["weight_decay"] if weight_decay is None else weight_decay
        self.max_grad_norm = c["max_grad_norm"] if max_grad_norm is None else max_grad_norm
        self.beta1, self.beta2 = betas
        self.eps = eps
        st = model.store
        self.master = st.flat.float()
        self.m = torch.zeros_like(self.master)
        self.v = torch.zeros_like(self.master)
        self.acc = c["accumulation_steps"]
        self.grad32 = torch.zeros_like(self.master) if self.acc > 1 else None
        self.rep32 = torch.zeros(st.total - st.sharded_end, dtype=torch.float32, device=st.flat.device)
        self.norm2 = torch.zeros((), dtype=torch.float64, device=st.flat.device)
        self.loss_sum = torch.zeros((), dtype=torch.float32, device=st.flat.device)
        self.step_count = 0

    def step(self, batches):
        """One optimizer step over `batches` = [(tokens, labels)] * accumulation_steps.
        Returns device tensors (mean loss, squared global grad norm)."""
        model, st = self.model, self.model.store
        if len(batches) != self.acc:
            raise ValueError(f"expected {self.acc} micro-batches")
        self.loss_sum.zero_()
        for mb, (tokens, labels) in enumerate(batches):
            with tracing.scope(f"trainer.micro_batch{mb}"):
                loss = model.forward_backward(tokens, labels, loss_scale=1.0 / self.acc)
                self.loss_sum.add_(loss.reshape(()) / self.acc)
                if self.grad32 is not None:
                    self.grad32.add_(st.grad)
        with tracing.scope("trainer.optimizer"):
            self._optimizer_step()
        return self.loss_sum, self.norm2

    def _optimizer_step(self):
        """Replicated-gradient all-reduce, global norm (FP64, replicated counted
        once), clipped FP32-master AdamW on sharded and replicated parameters."""
        model, st = self.model, self.model.store
        sh = st.sharded_end
        if self.grad32 is not None:
            sharded = self.grad32[:sh]
            self.rep32.copy_(self.grad32[sh:])
        else:
            sharded = st.grad[:sh]
            self.rep32.copy_(st.grad[sh:])
        tp = model.tp
        tp.all_reduce(self.rep32)
        O.sqsum(sharded, self.norm2)
        if model.rank == 0:
            O.sqsum(self.rep32, self.norm2, accumulate=True)
        tp.all_reduce(self.norm2)
        self.step_count += 1
        common = dict(max_norm=self.max_grad_norm, lr=self.lr, weight_decay=self.weight_decay,
                      beta1=self.beta1, beta2=self.beta2, eps=self.eps, step=self.step_count)
        O.adamw(self.master[:sh], self.m[:sh], self.v[:sh], sharded, st.flat[:sh], st.sharded_decay_end,
                self.norm2, **common)
        O.adamw(self.master[sh:], self.m[sh:], self.v[sh:], self.rep32, st.flat[sh:],
                st.replicated_decay_end - sh, self.norm2, **common)
        if self.grad32 is not None:
            self.grad32.zero_()

    def train_step(self, host_batches):
        """Public one-call step: copies each micro-batch's (tokens, labels) from
        (pinned) host memory to the device, runs `step`, and returns host floats
        (mean loss, global grad norm)."""
        dev = self.model.device
        batches = [(t.to(dev, non_blocking=True), l.to(dev, non_blocking=True)) for t, l in host_batches]
        return self.step_host(batches)

    def step_host(self, batches):
        """`step` plus one device->host read of (loss, grad norm); raises if non-finite."""
        loss, norm2 = self.step(batches)
        values = torch.stack([loss.double(), norm2]).cpu()
        if self.model.device.type == "cuda":
            check_status(self.model.device)
        lv, n2 = float(values[0]), float(values[1])
        if not math.isfinite(lv) or not math.isfinite(n2):
            raise RuntimeError("non-finite loss or global gradient norm")
        return lv, math.sqrt(n2)
