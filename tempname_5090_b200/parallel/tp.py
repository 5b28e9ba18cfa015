"""Tensor/sequence-parallel primitives used by the GPT model.

    ag_linear   column-parallel linear on a sequence-parallel shard:
                gather_rows(x) @ W^T  (+bias, GeLU / GeLU-backward epilogues)
    linear_rs   row-parallel linear into a sequence-parallel shard:
                scatter_sum(x @ W^T)  (+ residual + bias), ordered BF16 sum
    gather_rows / scatter_sum / all_reduce  plain collectives

On CUDA with W > 1 the two linears are the fused NVLink kernels (AGGemm,
GemmRS).  With W = 1 they are local tcgen05 GEMMs with the same epilogues.
Transport `nccl_plain` is the unfused control: the same tcgen05 GEMMs with a
plain NCCL all_gather_into_tensor before / reduce_scatter_tensor after them
(NCCL's own reduction order, residual and bias added afterwards) -- the
"library collectives around our GEMMs" step the fused operators must beat.
On CPU tensors (gloo process groups, unit tests) they are written with
torch.distributed collectives and the reference arithmetic, including the
ordered "round to BF16 after every source" reduction, so a CPU run of the
model is the oracle of the GPU run.
Semantics: ColumnLinear / RowLinear / SumScatter of TempName-5090
python/flux_5090/model.py:75-141.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops import gemm as G
from ..ops import taco


class TensorParallel:
    def __init__(self, group=None, *, arm: str = "flux", transport: str = "nvlink",
                 chunk_rows: int = 128, plans: dict | None = None, timeout_ns: int = 10_000_000_000):
        # group="local": a single-rank context even inside an initialised job.
        local = isinstance(group, str) and group == "local"
        self.group = None if local else group
        self.initialized = (not local) and dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(self.group) if self.initialized else 1
        self.rank = dist.get_rank(self.group) if self.initialized else 0
        self.arm, self.transport, self.chunk_rows = arm, transport, chunk_rows
        self.plans = plans or {}
        self.timeout_ns = timeout_ns
        self._ag: dict = {}
        self._rs: dict = {}

    # ------------------------------------------------------------ helpers
    def _cuda_multi(self, t: torch.Tensor) -> bool:
        return t.is_cuda and self.world > 1

    def gather_rows(self, x: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return x.contiguous()
        out = torch.empty((x.shape[0] * self.world, *x.shape[1:]), dtype=x.dtype, device=x.device)
        if x.is_cuda:
            dist.all_gather_into_tensor(out, x.contiguous(), group=self.group)
        else:
            pieces = list(out.chunk(self.world))
            dist.all_gather(pieces, x.contiguous(), group=self.group)
            out = torch.cat(pieces)
        return out

    def scatter_sum(self, x: torch.Tensor) -> torch.Tensor:
        """Reduce-scatter by rows (the embedding's SumScatter): the pull
        transport's reducer CTAs over NVLink, NCCL for the unfused transports."""
        if self.world == 1:
            return x.contiguous()
        M, N = x.shape
        if x.is_cuda and self.transport == "nvlink" and self.arm == "flux" and M % (128 * self.world) == 0 \
                and N % 256 == 0:
            return self.rs_operator(M, N, 8, "embed").scatter(x.contiguous())
        if x.is_cuda:
            out = torch.empty((x.shape[0] // self.world, *x.shape[1:]), dtype=x.dtype, device=x.device)
            dist.reduce_scatter_tensor(out, x.contiguous(), group=self.group)
            return out
        copy = x.contiguous().clone()
        dist.all_reduce(copy, group=self.group)
        return copy.chunk(self.world)[self.rank].contiguous()

    def all_reduce(self, x: torch.Tensor, op=None) -> torch.Tensor:
        if self.world > 1:
            dist.all_reduce(x, op=dist.ReduceOp.SUM if op is None else op, group=self.group)
        return x

    # ------------------------------------------------------- fused linears
    def ag_operator(self, site, m: int, k: int, n: int | None = None):
        """The AG->GEMM operator of a call site (its gather buffer is the saved
        input of that site); `n` (the GEMM's N) sizes its communication CTAs."""
        from .ag_gemm import AGGemm
        if site not in self._ag:
            self._ag[site] = AGGemm(m, k, self.group, timeout_ns=self.timeout_ns, n=n)
        return self._ag[site]

    def ag_input(self, site, m: int, k: int, n: int, on_cuda: bool):
        """Where the producer of `site`'s next AG->GEMM input should write it:
        this rank's chunk of the fused operator's gather buffer (written in
        place, it is published to the peers without a copy), or None (one rank,
        CPU, or an unfused transport)."""
        if self.world == 1 or not on_cuda or self.transport != "nvlink":
            return None
        return self.ag_operator(site, m, k, n).input_buffer()

    def ag_linear(self, site, shard: torch.Tensor, weight: torch.Tensor, *, b_mn: bool = False,
                  bias=None, gelu_aux=None, gelu_grad_of=None, out=None):
        """Return (output [M, N], gathered input [M, K])."""
        if self.world == 1:
            y = G.matmul(shard, weight, b_t=b_mn, bias=bias, gelu_aux=gelu_aux,
                         gelu_grad_of=gelu_grad_of, out=out)
            return y, shard
        if shard.is_cuda and self.transport == "nccl_plain":
            full = self.gather_rows(shard)
            y = G.matmul(full, weight, b_t=b_mn, bias=bias, gelu_aux=gelu_aux, gelu_grad_of=gelu_grad_of, out=out)
            return y, full
        if shard.is_cuda:
            op = self.ag_operator(site, shard.shape[0] * self.world, shard.shape[1],
                                  weight.shape[1] if b_mn else weight.shape[0])
            y = op.forward(shard, weight, b_mn=b_mn, bias=bias, gelu_aux=gelu_aux,
                           gelu_grad_of=gelu_grad_of, out=out)
            return y, op.gathered
        full = self.gather_rows(shard)
        y = G.matmul(full, weight, b_t=b_mn, bias=bias, gelu_aux=gelu_aux, gelu_grad_of=gelu_grad_of, out=out)
        return y, full

    def rs_operator(self, m: int, n: int, k: int, role: str):
        from .gemm_rs import GemmRS, RSWorkspace
        key = (m, n, role)
        if key not in self._rs:
            ws = self._rs.get(("ws", m, n))
            plan = self.plans.get(role) if self.arm.endswith("arrival") else None
            if plan is None and self.arm.endswith("arrival"):
                from .planning import make_role
                plan = make_role(m, n, k, self.world, self.chunk_rows)
            op = GemmRS(m, n, k, self.group, arm=self.arm, chunk_rows=self.chunk_rows, plan=plan,
                        transport=self.transport, timeout_ns=self.timeout_ns, workspace=ws)
            self._rs[("ws", m, n)] = op.workspace
            self._rs[key] = op
        return self._rs[key]

    def linear_rs(self, full: torch.Tensor, weight: torch.Tensor, *, b_mn: bool = False, residual=None,
                  bias=None, role: str = "mlp", out=None) -> torch.Tensor:
        """scatter_sum(full @ W^T) (+ residual, + bias) -> [M/W, N]."""
        if self.world == 1:
            return G.matmul(full, weight, b_t=b_mn, residual=residual, bias=bias, out=out)
        M = full.shape[0]
        N = weight.shape[1] if b_mn else weight.shape[0]
        if full.is_cuda and self.transport == "nccl_plain":
            partial = G.matmul(full, weight, b_t=b_mn)
            y = self.scatter_sum(partial)
            if residual is not None or bias is not None:
                z = y.float()
                if residual is not None:
                    z = (residual.float() + z).to(torch.bfloat16).float()
                if bias is not None:
                    z = z + bias.float()
                y = z.to(torch.bfloat16)
            if out is not None:
                out.copy_(y)
                return out
            return y
        if full.is_cuda:
            op = self.rs_operator(M, N, full.shape[1], role)
            return op.forward(full, weight, b_mn=b_mn, residual=residual, bias=bias, out=out)
        partial = G.matmul(full, weight, b_t=b_mn)
        parts = [torch.empty_like(partial) for _ in range(self.world)]
        dist.all_gather(parts, partial, group=self.group)
        rows = M // self.world
        mine = [p[self.rank * rows:(self.rank + 1) * rows] for p in parts]
        if self.arm != "flux":
            # quantized arms: every remote source passes through the TACO codec
            mine = [m if s == self.rank else taco.decode_cpu(taco.encode_cpu(m), m.numel()).reshape(m.shape)
                    for s, m in enumerate(mine)]
        y = taco.ordered_sum_cpu(mine)
        if residual is not None:
            y = (residual.float() + y.float()).to(torch.bfloat16)
        if bias is not None:
            y = (y.float() + bias.float()).to(torch.bfloat16)
        if out is not None:
            out.copy_(y)
            return out
        return y

    def close(self):
        for op in list(self._ag.values()):
            op.close()
        for key, op in list(self._rs.items()):
            if key[0] != "ws":
                op.close()
        self._ag.clear()
        self._rs.clear()
