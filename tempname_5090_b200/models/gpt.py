"""Tensor/sequence-parallel GPT (pre-LN, exact GeLU, tied embedding) for B200.

Parameter names, per-rank shapes, sharding and initialisation reproduce
TempName-5090 python/flux_5090/model.py:178-229 (state_dict layout):

    embedding [V/W, h] (tied LM head)        position [S, h] (replicated)
    layers.i.{ln1,ln2}_{weight,bias} [h]     layers.i.qkv_weight [3h/W, h], qkv_bias [3h/W]
    layers.i.attn_weight [h, h/W]            layers.i.attn_bias [h] (replicated)
    layers.i.fc1_weight [f/W, h], fc1_bias [f/W]
    layers.i.fc2_weight [h, f/W]             layers.i.fc2_bias [h] (replicated)
    final_weight / final_bias [h]

Seeds are name-derived (seed + sha256(tag)[:8] + 1000003*rank for sharded
tensors), std 0.02 (0.02/sqrt(2L) for attn/fc2 weights), LN weights 1, biases 0.

Unlike the reference (torch autograd over custom Functions), the training
program here is explicit: `forward_backward` runs the forward with the fused
AG->GEMM / GEMM->RS operators, saves exactly the activations the backward
needs, and writes every gradient straight into one flat BF16 gradient buffer
(weight gradients are tcgen05 GEMM outputs, no extra copies).  Forward
arithmetic order matches the reference: value = (value + RowLinear(...)) + bias.
All parameters live in one flat BF16 buffer ordered [sharded matrices |
sharded vectors | replicated matrices | replicated vectors] so the optimizer
is two fused launches.
"""
from __future__ import annotations

import hashlib
import math
from dataclasses import dataclass

import torch

from ..config import parameter_counts, validate_config
from ..ops import attention as A
from ..ops import embedding as E
from ..ops import gemm as G
from ..ops import loss as CE
from ..ops import norm as N
from ..parallel.tp import TensorParallel
from ..utils import tracing

ALIGN = 64  # elements; keeps every parameter view 128-byte aligned


@dataclass
class ParamSpec:
    name: str
    shape: tuple
    replicated: bool
    init: str          # "normal" | "one" | "zero"
    std: float
    tag: str

    @property
    def numel(self) -> int:
        n = 1
        for s in self.shape:
            n *= s
        return n

    @property
    def matrix(self) -> bool:
        return len(self.shape) >= 2


def param_specs(c: dict, world: int) -> list:
    h, f, V, S, L = c["hidden"], c["ffn"], c["vocab"], c["sequence"], c["layers"]
    specs = [ParamSpec("embedding", (V // world, h), False, "normal", 0.02, "embedding"),
             ParamSpec("position", (S, h), True, "normal", 0.02, "position")]
    small = 0.02 / math.sqrt(2 * L)
    for i in range(L):
        p = f"layers.{i}"
        for norm in ("ln1", "ln2"):
            specs.append(ParamSpec(f"{p}.{norm}_weight", (h,), True, "one", 0.0, f"{p}{norm}w"))
            specs.append(ParamSpec(f"{p}.{norm}_bias", (h,), True, "zero", 0.0, f"{p}{norm}b"))
        specs += [
            ParamSpec(f"{p}.qkv_weight", (3 * h // world, h), False, "normal", 0.02, f"{p}qkvw"),
            ParamSpec(f"{p}.qkv_bias", (3 * h // world,), False, "zero", 0.0, f"{p}qkvb"),
            ParamSpec(f"{p}.attn_weight", (h, h // world), False, "normal", small, f"{p}attnw"),
            ParamSpec(f"{p}.attn_bias", (h,), True, "zero", 0.0, f"{p}attnb"),
            ParamSpec(f"{p}.fc1_weight", (f // world, h), False, "normal", 0.02, f"{p}fc1w"),
            ParamSpec(f"{p}.fc1_bias", (f // world,), False, "zero", 0.0, f"{p}fc1b"),
            ParamSpec(f"{p}.fc2_weight", (h, f // world), False, "normal", small, f"{p}fc2w"),
            ParamSpec(f"{p}.fc2_bias", (h,), True, "zero", 0.0, f"{p}fc2b"),
        ]
    specs.append(ParamSpec("final_weight", (h,), True, "one", 0.0, "final_ln_w"))
    specs.append(ParamSpec("final_bias", (h,), True, "zero", 0.0, "final_ln_b"))
    return specs


def _round_up(x: int) -> int:
    return (x + ALIGN - 1) // ALIGN * ALIGN


class ParamStore:
    """Flat BF16 parameters and gradients with named views and optimizer regions."""

    def __init__(self, specs, device, rank: int, seed: int, dtype=torch.bfloat16, init: bool = True):
        self.specs = specs
        self.device = torch.device(device)
        groups = [[s for s in specs if not s.replicated and s.matrix],
                  [s for s in specs if not s.replicated and not s.matrix],
                  [s for s in specs if s.replicated and s.matrix],
                  [s for s in specs if s.replicated and not s.matrix]]
        self.offsets = {}
        off = 0
        bounds = []
        for g in groups:
            for s in g:
                self.offsets[s.name] = off
                off += _round_up(s.numel)
            bounds.append(off)
        self.total = off
        self.sharded_end = bounds[1]
        self.sharded_decay_end = bounds[0]
        self.replicated_decay_end = bounds[2]
        self.flat = torch.zeros(self.total, dtype=dtype, device=self.device)
        self.grad = torch.zeros(self.total, dtype=dtype, device=self.device)
        self.params = {}
        self.grads = {}
        for s in specs:
            o = self.offsets[s.name]
            self.params[s.name] = self.flat[o:o + s.numel].view(s.shape)
            self.grads[s.name] = self.grad[o:o + s.numel].view(s.shape)
        self.replicated = {s.name for s in specs if s.replicated}
        if init:
            self.initialize(rank, seed)

    def initialize(self, rank: int, seed: int) -> None:
        for s in self.specs:
            t = self.params[s.name]
            if s.init == "one":
                t.fill_(1)
            elif s.init == "zero":
                t.zero_()
            else:
                salt = int.from_bytes(hashlib.sha256(s.tag.encode()).digest()[:8], "little")
                g = torch.Generator(device=self.device)
                g.manual_seed((seed + salt + (0 if s.replicated else 1000003 * rank)) % (2 ** 63 - 1))
                t.normal_(0, s.std, generator=g)

    def named_parameters(self):
        return [(s.name, self.params[s.name]) for s in self.specs]

    def numel(self) -> int:
        return sum(s.numel for s in self.specs)


class GPT:
    """TP/SP GPT over `TensorParallel`; one instance per rank."""

    def __init__(self, config: dict, arm: str = "flux", group=None, device="cuda", seed: int = 1234,
                 transport: str = "nvlink", execution_plan: dict | None = None, init: bool = True,
                 timeout_ns: int = 10_000_000_000):
        plans = None
        if execution_plan is not None:
            plans = execution_plan.get("roles", execution_plan)
        self.tp = TensorParallel(group, arm=arm, transport=transport, chunk_rows=int(config.get("chunk_rows", 128)),
                                 plans=plans, timeout_ns=timeout_ns)
        self.world, self.rank = self.tp.world, self.tp.rank
        self.config = validate_config(config, self.world)
        self.arm = arm
        self.device = torch.device(device)
        self.seed = seed
        self.specs = param_specs(self.config, self.world)
        self.store = ParamStore(self.specs, self.device, self.rank, seed, init=init)
        self.p = self.store.params
        self.g = self.store.grads
        self.forward_calls = 0
        c = self.config
        self.M = c["sequence"] * c["micro_batch"]
        self.Ml = self.M // self.world
        self.h, self.f = c["hidden"], c["ffn"]
        self.lh = c["heads"] // self.world
        self.Vl = c["vocab"] // self.world
        self.eps = c["layer_norm_epsilon"]
        counts = parameter_counts(c, self.world)
        if self.store.numel() != counts["parameters_per_rank"]:
            raise RuntimeError("parameter count differs from the configuration")
        self._ws = {}

    # --------------------------------------------------------------- state
    def named_parameters(self):
        return self.store.named_parameters()

    def parameters(self):
        return [t for _, t in self.named_parameters()]

    def state_dict(self) -> dict:
        return {name: t for name, t in self.named_parameters()}

    def load_state_dict(self, state: dict) -> None:
        names = [n for n, _ in self.named_parameters()]
        if set(state) != set(names):
            raise ValueError("state_dict keys differ from the model's parameters")
        for name in names:
            src = state[name]
            if tuple(src.shape) != tuple(self.p[name].shape):
                raise ValueError(f"shape mismatch for {name}")
            self.p[name].copy_(src)

    def _workspace(self, name, numel, dtype):
        t = self._ws.get(name)
        if t is None or t.numel() < numel or t.dtype != dtype:
            t = torch.empty(numel, dtype=dtype, device=self.device)
            self._ws[name] = t
        return t

    # ------------------------------------------------------------- forward
    def _forward(self, tokens, targets, keep: bool, loss_scale: float):
        c, tp = self.config, self.tp
        M, Ml, h, lh = self.M, self.Ml, self.h, self.lh
        if tokens.shape != (M,) or targets.shape != (M,):
            raise ValueError("tokens/targets must hold the full flattened micro-batch")
        start = self.rank * self.Vl
        row0 = self.rank * Ml
        contrib = E.lookup(tokens, self.p["embedding"], start)
        x = tp.scatter_sum(contrib)
        E.add_position(x, self.p["position"], row0)
        saved = []
        for i in range(c["layers"]):
            with tracing.scope(f"gpt.layer{i}.forward"):
                x = self._layer_forward(i, x, saved, keep)
        x_final = x
        buf = tp.ag_input(("head", 0), M, self.h, self.Vl, x.is_cuda)
        lnf, meanf, rstdf = N.layer_norm_fwd(x_final, self.p["final_weight"], self.p["final_bias"], self.eps, out=buf)
        logits, lnf_full = tp.ag_linear(("head", 0), lnf, self.p["embedding"])
        loss, ce_state = CE.forward(logits, targets, tp.group, self.rank, self.world, scale=loss_scale / M)
        self.forward_calls += 1
        tape = (tokens, targets, saved, x_final, meanf, rstdf, lnf_full, logits, ce_state) if keep else None
        return loss, tape

    def _layer_forward(self, i, x, saved, keep):
        """One transformer block forward (pre-LN); appends its tape when `keep`."""
        c, tp, M = self.config, self.tp, self.M
        lh = self.lh
        p = f"layers.{i}."
        x_in = x
        # LayerNorm outputs are written straight into the fused AG->GEMM's gather
        # buffer (published to the peers without a copy) when TP > 1.
        h, W = self.h, self.world
        buf = tp.ag_input(("qkv", i), M, h, 3 * h // W, x.is_cuda)
        ln1, mean1, rstd1 = N.layer_norm_fwd(x_in, self.p[p + "ln1_weight"], self.p[p + "ln1_bias"], self.eps,
                                             out=buf)
        qkv, ln1_full = tp.ag_linear(("qkv", i), ln1, self.p[p + "qkv_weight"], bias=self.p[p + "qkv_bias"])
        attn, lse = A.forward(qkv, c["micro_batch"], c["sequence"], lh)
        x2 = tp.linear_rs(attn, self.p[p + "attn_weight"], residual=x_in, bias=self.p[p + "attn_bias"],
                          role="attn")
        buf = tp.ag_input(("fc1", i), M, h, self.f // W, x.is_cuda)
        ln2, mean2, rstd2 = N.layer_norm_fwd(x2, self.p[p + "ln2_weight"], self.p[p + "ln2_bias"], self.eps,
                                             out=buf)
        pre = torch.empty((M, self.f // self.world), dtype=torch.bfloat16, device=self.device)
        act, ln2_full = tp.ag_linear(("fc1", i), ln2, self.p[p + "fc1_weight"], bias=self.p[p + "fc1_bias"],
                                     gelu_aux=pre)
        x = tp.linear_rs(act, self.p[p + "fc2_weight"], residual=x2, bias=self.p[p + "fc2_bias"], role="mlp")
        if keep:
            saved.append((x_in, mean1, rstd1, ln1_full, qkv, attn, lse, x2, mean2, rstd2, ln2_full, pre, act))
        return x

    def _layer_backward(self, i, tape, dx, ln_ws, col_ws):
        """One transformer block backward: writes its parameter gradients and
        returns the gradient of its input."""
        c, tp, g = self.config, self.tp, self.g
        p = f"layers.{i}."
        (x_in, mean1, rstd1, ln1_full, qkv, attn, lse, x2, mean2, rstd2, ln2_full, pre, act) = tape
        # fc2 (row-parallel): x = x2 + RS(act @ Wfc2^T) + b
        N.column_sum(dx, out=g[p + "fc2_bias"], workspace=col_ws)
        dpre, dfull = tp.ag_linear(("fc2_bwd", i % 2), dx, self.p[p + "fc2_weight"], b_mn=True,
                                   gelu_grad_of=pre)
        G.matmul(dfull, act, a_t=True, b_t=True, out=g[p + "fc2_weight"])
        # fc1 (column-parallel): pre = gather(ln2) @ Wfc1^T + b
        N.column_sum(dpre, out=g[p + "fc1_bias"], workspace=col_ws)
        dln2 = tp.linear_rs(dpre, self.p[p + "fc1_weight"], b_mn=True, role="mlp_bwd")
        G.matmul(dpre, ln2_full, a_t=True, b_t=True, out=g[p + "fc1_weight"])
        M, h, W = self.M, self.h, self.world
        dx2, dw2, db2 = N.layer_norm_bwd(dln2, x2, self.p[p + "ln2_weight"], mean2, rstd2, dres=dx,
                                         workspace=ln_ws,
                                         out=tp.ag_input(("attn_bwd", i % 2), M, h, h // W, dx.is_cuda))
        g[p + "ln2_weight"].copy_(dw2)
        g[p + "ln2_bias"].copy_(db2)
        # attention out-projection (row-parallel): x2 = x_in + RS(attn @ Wattn^T) + b
        N.column_sum(dx2, out=g[p + "attn_bias"], workspace=col_ws)
        dattn, dfull2 = tp.ag_linear(("attn_bwd", i % 2), dx2, self.p[p + "attn_weight"], b_mn=True)
        G.matmul(dfull2, attn, a_t=True, b_t=True, out=g[p + "attn_weight"])
        dqkv = A.backward(qkv, attn, dattn, lse, c["micro_batch"], c["sequence"], self.lh)
        # QKV (column-parallel)
        N.column_sum(dqkv, out=g[p + "qkv_bias"], workspace=col_ws)
        dln1 = tp.linear_rs(dqkv, self.p[p + "qkv_weight"], b_mn=True, role="attn_bwd")
        G.matmul(dqkv, ln1_full, a_t=True, b_t=True, out=g[p + "qkv_weight"])
        # The input gradient feeds the previous layer's FC2-backward AG->GEMM.
        nxt = tp.ag_input(("fc2_bwd", (i - 1) % 2), M, h, self.f // W, dx2.is_cuda) if i > 0 else None
        dx, dw1, db1 = N.layer_norm_bwd(dln1, x_in, self.p[p + "ln1_weight"], mean1, rstd1, dres=dx2,
                                        workspace=ln_ws, out=nxt)
        g[p + "ln1_weight"].copy_(dw1)
        g[p + "ln1_bias"].copy_(db1)
        return dx

    @torch.no_grad()
    def loss(self, tokens, targets) -> torch.Tensor:
        """Mean cross-entropy of one micro-batch (forward only)."""
        loss, _ = self._forward(tokens, targets, keep=False, loss_scale=1.0)
        return loss

    # ------------------------------------------------------------ backward
    @torch.no_grad()
    def forward_backward(self, tokens, targets, loss_scale: float = 1.0) -> torch.Tensor:
        """Forward + backward of one micro-batch; gradients of `loss * loss_scale`
        are written into `self.store.grad`.  Returns the (unscaled) mean loss."""
        loss, tape = self._forward(tokens, targets, keep=True, loss_scale=1.0)
        self._backward(tape, loss_scale)
        return loss

    def _backward(self, tape, loss_scale: float):
        c, tp = self.config, self.tp
        tokens, targets, saved, x_final, meanf, rstdf, lnf_full, logits, ce_state = tape
        M = self.M
        start = self.rank * self.Vl
        g = self.g
        ln_ws = self._workspace("ln", 2 * 64 * self.h, torch.float32)
        col_ws = self._workspace("col", 64 * max(self.f // self.world, 3 * self.h // self.world, self.h),
                                 torch.float32)
        # Cross-entropy -> dlogits (in place), LM head (tied embedding)
        CE.backward(logits, targets, ce_state, loss_scale / M)
        dlnf = tp.linear_rs(logits, self.p["embedding"], b_mn=True, role="head")
        G.matmul(logits, lnf_full, a_t=True, b_t=True, out=g["embedding"])
        L = c["layers"]
        dx, dwf, dbf = N.layer_norm_bwd(dlnf, x_final, self.p["final_weight"], meanf, rstdf, workspace=ln_ws,
                                        out=tp.ag_input(("fc2_bwd", (L - 1) % 2), M, self.h, self.f // self.world,
                                                        dlnf.is_cuda))
        g["final_weight"].copy_(dwf)
        g["final_bias"].copy_(dbf)
        for i in reversed(range(c["layers"])):
            with tracing.scope(f"gpt.layer{i}.backward"):
                dx = self._layer_backward(i, saved[i], dx, ln_ws, col_ws)
        # value = scatter_sum(embedding contributions) + position
        E.position_grad(dx, c["sequence"], self.rank * self.Ml, out=g["position"])
        dcontrib = tp.gather_rows(dx)
        E.lookup_grad(tokens, dcontrib, g["embedding"], start, accumulate=True)

    def close(self):
        self.tp.close()
