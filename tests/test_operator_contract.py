"""Host-side contract of the fused operators (GemmRS, AG->GEMM), on CPU.

1. NVLink transport with a recording stand-in for the native module: per call
   exactly one producer launch then one receiver launch, both with the call's
   epoch and the same receive-slot parity; mode and consumer policy per arm; the
   rotated production order and the unrotated consumer order; a failed launch
   poisons the operator (later calls raise and launch nothing).
2. NCCL transport (the reference mechanism: one GEMM, per-block sparse
   all_to_all on two lane groups, ordered (decode+)reduce) on two Gloo ranks:
   bitwise equal to the ordered BF16 sum of the sources' partials, with remote
   blocks through the TACO codec in the quantized arm.
3. AG->GEMM with a recording stand-in: cumulative chunk-flag targets (every
   CTA of every call bumps each owner's counter once), epilogue bits, own row
   chunk first in the tile order, shard-shape checks.
"""
import os
import socket
import tempfile

import pytest
import torch

M, N, K, CHUNK = 512, 512, 64, 128


class _Buf:
    """Stand-in for a symmetric buffer: a device-pointer table and a local pointer."""

    def __init__(self, tag):
        self.ptrs = torch.tensor([tag, tag + 1], dtype=torch.int64)
        self.local = tag


class _FakeLib:
    def __init__(self):
        self.calls = []
        self.fail_push = False

    def gemm_rs_push(self, x, a_mn, w, b_mn, mode, recv_ptrs, flag_ptrs, rank, world, chunk_rows, epoch,
                     slot_bytes, tile_order, status, timeout_ns, max_ctas, delay_tile, delay_ns):
        if self.fail_push:
            raise RuntimeError("injected launch failure")
        self.calls.append(("push", dict(mode=mode, recv=recv_ptrs, flags=flag_ptrs, epoch=epoch,
                                        order=tile_order.tolist(), rank=rank, world=world,
                                        delay=(delay_tile, delay_ns), slot=slot_bytes, chunk=chunk_rows)))

    def gemm_rs_pull(self, x, a_mn, w, b_mn, partial_local, partial_ptrs, flag_ptrs, my_flags, rank, world, epoch,
                     tile_order, consumer_order, out, residual, bias, status, timeout_ns, comm_ctas, phase, stamps,
                     produced, delay_tile, delay_ns, max_ctas, cta_stamps, pair):
        if self.fail_push:
            raise RuntimeError("injected launch failure")
        self.calls.append(("pull", dict(partial=partial_local, partials=partial_ptrs, flags=flag_ptrs,
                                        my_flags=my_flags, epoch=epoch, order=tile_order.tolist(),
                                        consumer=consumer_order.tolist(), rank=rank, world=world,
                                        comm_ctas=comm_ctas, phase=phase, residual=residual is not None,
                                        bias=bias is not None, delay=(delay_tile, delay_ns))))

    def rs_reduce(self, recv, flags, slot_bytes, rank, world, rows, n, tile_n, chunk_rows, quantized, epoch,
                  out, residual, bias, order, arrival, claims, status, timeout_ns, max_ctas, stamps):
        self.calls.append(("reduce", dict(recv=recv, flags=flags, epoch=epoch, quantized=quantized,
                                          arrival=arrival, claims=claims is not None, order=order.tolist(),
                                          residual=residual is not None, bias=bias is not None,
                                          slot=slot_bytes, chunk=chunk_rows)))


@pytest.mark.parametrize("arm", ["flux", "flux_taco", "flux_taco_interleaved", "flux_taco_interleaved_arrival"])
@pytest.mark.parametrize("rank,world", [(0, 2), (1, 2), (2, 4)])
def test_nvlink_transport_launch_contract(monkeypatch, arm, rank, world):
    from tempname_5090_b200.parallel import gemm_rs, mapping, planning
    fake = _FakeLib()
    monkeypatch.setattr(gemm_rs, "lib", lambda: fake)
    monkeypatch.setattr(gemm_rs, "count_launch", lambda n=1: None)
    plan = planning.make_role(M, N, K, world, CHUNK) if arm.endswith("arrival") else None
    recv, flags = [_Buf(100), _Buf(200)], _Buf(300)
    op = gemm_rs.GemmRS(M, N, K, arm=arm, chunk_rows=CHUNK, plan=plan,
                        _emulate=(rank, world, recv, flags), device="cpu")
    x = torch.zeros((M, K), dtype=torch.bfloat16)
    w = torch.zeros((N, K), dtype=torch.bfloat16)
    quantized = arm in mapping.QUANTIZED_ARMS
    consumer = mapping.consumer_tile_order(M, N, K, world, CHUNK, arm, rank, plan, 256)
    if not quantized:
        # BF16 arm: the pull transport, ONE launch per call (GEMM + reducer CTAs),
        # destinations interleaved one tile at a time starting with rank+1.
        production = mapping.pull_production_ids(M, N, K, world, CHUNK, arm, rank, plan, tile_n=256)
        tiles_n = N // 256
        per_dest = M // world // 128
        assert [tid // tiles_n // per_dest for tid in production[:world]] == [(rank + 1 + j) % world
                                                                              for j in range(world)]
        assert sorted(production) == list(range(len(production)))
        for call in range(1, 5):
            out = op.forward(x, w, residual=torch.zeros((M // world, N), dtype=torch.bfloat16))
            assert out.shape == (M // world, N) and len(fake.calls) == call
            kind, c = fake.calls[-1]
            assert kind == "pull" and c["phase"] == 6 and c["epoch"] == call
            assert c["partial"] == recv[call & 1].local and c["partials"] == recv[call & 1].ptrs.data_ptr()
            assert c["flags"] == flags.ptrs.data_ptr() and c["my_flags"] == flags.local
            assert c["order"] == production and c["consumer"] == consumer
            assert c["residual"] and not c["bias"] and c["delay"] == (-1, 0) and c["comm_ctas"] == op.comm_ctas
        fake.fail_push = True
        with pytest.raises(RuntimeError, match="injected"):
            op.forward(x, w)
        fake.fail_push = False
        before = len(fake.calls)
        with pytest.raises(RuntimeError, match="previously failed"):
            op.forward(x, w)
        assert len(fake.calls) == before and op.failed
        return
    production = mapping.linear_tile_ids(M, N, K, world, CHUNK, arm, plan, tile_n=256, shift=rank + 1)
    for call in range(1, 5):
        out = op.forward(x, w, residual=torch.zeros((M // world, N), dtype=torch.bfloat16))
        assert out.shape == (M // world, N)
        push, reduce = fake.calls[-2], fake.calls[-1]
        assert [push[0], reduce[0]] == ["push", "reduce"]
        assert len(fake.calls) == 2 * call  # one producer + one receiver launch per call
        p, r = push[1], reduce[1]
        assert p["epoch"] == r["epoch"] == call
        assert p["recv"] == recv[call & 1].ptrs.data_ptr() and r["recv"] == recv[call & 1].local
        assert p["flags"] == flags.ptrs.data_ptr() and r["flags"] == flags.local
        assert p["mode"] == (2 if quantized else 1) and r["quantized"] == quantized
        # both sides address the owner's two lane regions with the same layout
        lanes = mapping.PushLanes(M // world, N, CHUNK, world)
        assert p["slot"] == r["slot"] == lanes.lane_slot_bytes and p["chunk"] == r["chunk"] == CHUNK
        assert r["arrival"] == arm.endswith("arrival") and r["claims"] == arm.endswith("arrival")
        assert p["order"] == production and r["order"] == consumer
        assert r["residual"] and not r["bias"]
        assert p["delay"] == (-1, 0)  # the lane-skew diagnostic never fires in a normal call
    # A failed launch poisons the operator: no further launches.
    fake.fail_push = True
    with pytest.raises(RuntimeError, match="injected"):
        op.forward(x, w)
    fake.fail_push = False
    before = len(fake.calls)
    with pytest.raises(RuntimeError, match="previously failed"):
        op.forward(x, w)
    assert len(fake.calls) == before and op.failed


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _inputs(rank):
    g = torch.Generator().manual_seed(40 + rank)
    x = torch.randn((M, K), generator=g).to(torch.bfloat16)
    w = (0.1 * torch.randn((N, K), generator=g)).to(torch.bfloat16)
    return x, w


def _nccl_worker(rank, world, port, out_dir, arm):
    import torch.distributed as dist
    from tempname_5090_b200.parallel.gemm_rs import GemmRS
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        op = GemmRS(M, N, K, arm=arm, chunk_rows=CHUNK, transport="nccl", device="cpu")
        x, w = _inputs(rank)
        outs = [op.forward(x, w).clone() for _ in range(2)]
        torch.save(dict(outs=outs, state=op.state(), recv_shape=tuple(op.recv_blocks.shape),
                        send_shape=tuple(op.send_packets.shape)), os.path.join(out_dir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("arm", ["flux", "flux_taco"])
def test_nccl_transport_two_gloo_ranks_match_ordered_sum(arm):
    import torch.multiprocessing as mp
    from tempname_5090_b200.ops import taco
    from tempname_5090_b200.ops.gemm import matmul
    world = 2
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_nccl_worker, args=(world, _free_port(), d, arm), nprocs=world, join=True)
        res = [torch.load(os.path.join(d, f"rank{r}.pt")) for r in range(world)]
    partials = [matmul(*_inputs(s)) for s in range(world)]
    rows = M // world
    for r in range(world):
        sources = []
        for s in range(world):
            part = partials[s][r * rows:(r + 1) * rows]
            if arm == "flux_taco" and s != r:
                blocks = [taco.decode_cpu(taco.encode_cpu(part[b:b + CHUNK]), CHUNK * N)
                          for b in range(0, rows, CHUNK)]
                part = torch.cat(blocks).reshape(rows, N)
            sources.append(part.reshape(-1))
        want = taco.ordered_sum_cpu(sources).reshape(rows, N)
        for got in res[r]["outs"]:
            assert torch.equal(got, want)
        assert res[r]["state"]["calls"] == 2 and res[r]["state"]["reduction_order"] == list(range(world))
        per, pbytes = rows // CHUNK, CHUNK * N // 128 * 136
        if arm == "flux_taco":  # packets only: no BF16-sized remote storage
            assert res[r]["recv_shape"] == (per, world - 1, pbytes) and res[r]["send_shape"] == (M // CHUNK, pbytes)
        else:
            assert res[r]["recv_shape"] == (per, world - 1, CHUNK * N * 2) and res[r]["send_shape"][0] == 0


class _FakeAGLib:
    def __init__(self):
        self.calls = []

    def ag_gemm(self, shard, gather, w, b_mn, out, epi, bias, aux, gather_ptrs, published_ptrs, pulled_ptrs,
                published_local, pulled_local, ready, rank, world, epoch, pulled_target, ready_target,
                tile_order, status, timeout_ns, bn, comm_ctas, phase, cta_stamps, block_stamps, pair):
        self.calls.append(dict(epi=epi, rank=rank, world=world, epoch=epoch,
                               pulled=pulled_target, ready=ready_target, order=tile_order.tolist(),
                               bn=bn, b_mn=b_mn, aux=aux is not None, bias=bias is not None, ctrl=published_local,
                               pulled_local=pulled_local, gather_ptrs=gather_ptrs, comm_ctas=comm_ctas,
                               phase=phase))


class _AGBuf(_Buf):
    def __init__(self, tag, m=1, k=1):
        super().__init__(tag)
        self._m, self._k = m, k
        self.peers = [tag + 10 * r for r in range(8)]

    def local_view(self, shape, dtype, offset=0):
        return torch.zeros(shape, dtype=dtype)


@pytest.mark.parametrize("rank,world", [(0, 2), (3, 4), (5, 8)])
def test_ag_gemm_launch_contract(monkeypatch, rank, world):
    from tempname_5090_b200.parallel import ag_gemm
    from tempname_5090_b200.ops import gemm as G
    fake = _FakeAGLib()
    monkeypatch.setattr(ag_gemm, "lib", lambda: fake)
    monkeypatch.setattr(ag_gemm, "count_launch", lambda n=1: None)
    m, k, n = 128 * world * 2, 256, 1024
    gather, ctrl = _AGBuf(500), _AGBuf(600)
    op = ag_gemm.AGGemm(m, k, comm_ctas=7, _emulate=(rank, world, gather, ctrl), device="cpu")
    shard = torch.zeros((m // world, k), dtype=torch.bfloat16)
    w = torch.zeros((n, k), dtype=torch.bfloat16)
    aux = torch.zeros((m, n), dtype=torch.bfloat16)
    op.forward(shard, w, bias=torch.zeros(n, dtype=torch.bfloat16))
    op.forward(shard, w, gelu_aux=aux)
    op.forward(shard, w.t().contiguous(), b_mn=True, gelu_grad_of=aux)
    c = fake.calls
    # One launch per call; targets: (W-1) peers x 7 gatherer CTAs finished
    # reading per previous call (cumulative), and the per-block arrival flag
    # equal to the call's epoch.
    assert [x["epoch"] for x in c] == [1, 2, 3] and all(x["phase"] == 7 for x in c)
    assert [x["pulled"] for x in c] == [0, 7 * (world - 1), 14 * (world - 1)]
    pulled_offset, _ = ag_gemm.control_layout(m)
    assert pulled_offset % 256 == 0 and pulled_offset >= 4 * m // 128
    assert all(x["pulled_local"] == ctrl.local + pulled_offset for x in c)
    assert [x["ready"] for x in c] == [1, 2, 3]
    assert [x["epi"] for x in c] == [G.EPI_BIAS, G.EPI_GELU, G.EPI_GELU_BWD]
    assert [x["aux"] for x in c] == [False, True, True] and [x["b_mn"] for x in c] == [False, False, True]
    # Own chunk first, then rank+1, ...: the first tiles need no peer data.
    order = c[0]["order"]
    tiles_n = (n + c[0]["bn"] - 1) // c[0]["bn"]
    per = m // world // 128
    first_rows = {tid // tiles_n for tid in order[:per * tiles_n]}
    assert first_rows == set(range(rank * per, (rank + 1) * per))
    assert sorted(order) == list(range(len(order)))
    assert all(x["ctrl"] == ctrl.local and x["gather_ptrs"] == gather.ptrs.data_ptr() for x in c)
    with pytest.raises(ValueError):
        op.forward(torch.zeros((m // world + 128, k), dtype=torch.bfloat16), w)
    # Emulation phases: 1 opens a new epoch, 2 and 4 reuse it.
    op.forward(shard, w, phase=1)
    op.forward(shard, w, phase=2)
    op.forward(shard, w, phase=4)
    assert [x["epoch"] for x in c[3:]] == [4, 4, 4] and [x["phase"] for x in c[3:]] == [1, 2, 4]


@pytest.mark.parametrize("bad", ["x_rows", "x_dtype", "w_k", "w_layout", "residual", "bias", "out"])
def test_gemm_rs_rejects_mismatched_operands_before_launching(monkeypatch, bad):
    from tempname_5090_b200.parallel import gemm_rs
    fake = _FakeLib()
    monkeypatch.setattr(gemm_rs, "lib", lambda: fake)
    monkeypatch.setattr(gemm_rs, "count_launch", lambda n=1: None)
    world = 2
    op = gemm_rs.GemmRS(M, N, K, _emulate=(0, world, [_Buf(1), _Buf(2)], _Buf(3)), device="cpu")
    bf = torch.bfloat16
    args = dict(x=torch.zeros((M, K), dtype=bf), w=torch.zeros((N, K), dtype=bf))
    kw = {}
    if bad == "x_rows":
        args["x"] = torch.zeros((M + 128, K), dtype=bf)
    elif bad == "x_dtype":
        args["x"] = torch.zeros((M, K), dtype=torch.float32)
    elif bad == "w_k":
        args["w"] = torch.zeros((N, K + 8), dtype=bf)
    elif bad == "w_layout":
        kw["b_mn"] = True  # [N, K] passed where [K, N] is declared
    elif bad == "residual":
        kw["residual"] = torch.zeros((M, N), dtype=bf)
    elif bad == "bias":
        kw["bias"] = torch.zeros((N + 1,), dtype=bf)
    elif bad == "out":
        kw["out"] = torch.zeros((M // world, N + 256), dtype=bf)
    with pytest.raises(ValueError):
        op.forward(args["x"], args["w"], **kw)
    assert fake.calls == [] and not op.failed and op.epoch == 0


@pytest.mark.parametrize("bad", ["w_k", "bias", "bias_dtype", "aux", "dtype"])
def test_ag_gemm_rejects_mismatched_operands_before_launching(monkeypatch, bad):
    from tempname_5090_b200.parallel import ag_gemm
    fake = _FakeAGLib()
    monkeypatch.setattr(ag_gemm, "lib", lambda: fake)
    monkeypatch.setattr(ag_gemm, "count_launch", lambda n=1: None)
    world, m, k, n = 2, 512, 256, 512
    op = ag_gemm.AGGemm(m, k, _emulate=(0, world, _AGBuf(1), _AGBuf(2)), device="cpu")
    bf = torch.bfloat16
    shard, w, kw = torch.zeros((m // world, k), dtype=bf), torch.zeros((n, k), dtype=bf), {}
    if bad == "w_k":
        w = torch.zeros((n, k + 8), dtype=bf)
    elif bad == "bias":
        kw["bias"] = torch.zeros((n - 1,), dtype=bf)
    elif bad == "bias_dtype":
        kw["bias"] = torch.zeros((n,), dtype=torch.float32)
    elif bad == "aux":
        kw["gelu_aux"] = torch.zeros((m // world, n), dtype=bf)
    elif bad == "dtype":
        shard = shard.float()
    with pytest.raises(ValueError):
        op.forward(shard, w, **kw)
    assert fake.calls == [] and op.calls == 0


def test_role_plans_reach_their_operators(monkeypatch):
    """The arrival arm's calibrated plans are routed by role (attn / mlp); roles
    without a plan (other shapes) get the identity order; other arms get none."""
    from tempname_5090_b200.parallel import gemm_rs, planning
    from tempname_5090_b200.parallel.tp import TensorParallel
    made = []

    class Recorder:
        def __init__(self, m, n, k, group, *, arm, chunk_rows, plan, transport, timeout_ns, workspace):
            made.append(dict(m=m, n=n, k=k, arm=arm, plan=plan))
            self.workspace = object()
    monkeypatch.setattr(gemm_rs, "GemmRS", Recorder)
    world, m, h, f = 8, 2048, 4096, 16384
    orders = planning.candidates(m, h, h // world, world, 128)
    attn_plan = planning.make_role(m, h, h // world, world, 128, orders[1]["arrival_order"])
    mlp_plan = planning.make_role(m, h, f // world, world, 128)
    tp = TensorParallel(None, arm="flux_taco_interleaved_arrival", plans=dict(attn=attn_plan, mlp=mlp_plan))
    tp.world = world
    tp.rs_operator(m, h, h // world, "attn")
    tp.rs_operator(m, h, f // world, "mlp")
    tp.rs_operator(m, h, 3 * h // world, "attn_bwd")
    assert made[0]["plan"] is attn_plan and made[1]["plan"] is mlp_plan
    assert made[2]["plan"]["arrival_order"] == planning.base_order(m, h, 3 * h // world, world, 128)
    assert tp.rs_operator(m, h, h // world, "attn") is tp.rs_operator(m, h, h // world, "attn")  # cached
    made.clear()
    plain = TensorParallel(None, arm="flux_taco", plans=dict(attn=attn_plan))
    plain.world = world
    plain.rs_operator(m, h, h // world, "attn")
    assert made[0]["plan"] is None


@pytest.mark.parametrize("arm", ["flux", "flux_taco"])  # pull and push transports
def test_failure_poisons_every_operator_sharing_the_workspace(monkeypatch, arm):
    from tempname_5090_b200.parallel import gemm_rs
    fake = _FakeLib()
    monkeypatch.setattr(gemm_rs, "lib", lambda: fake)
    monkeypatch.setattr(gemm_rs, "count_launch", lambda n=1: None)
    recv, flags = [_Buf(1), _Buf(2)], _Buf(3)
    a = gemm_rs.GemmRS(M, N, K, arm=arm, _emulate=(0, 2, recv, flags), device="cpu")
    b = gemm_rs.GemmRS(M, N, 2 * K, arm=arm, _emulate=(0, 2, recv, flags), device="cpu")
    b.workspace = a.workspace  # two projections of one (M, N) share slots, flags and epochs
    x, w = torch.zeros((M, K), dtype=torch.bfloat16), torch.zeros((N, K), dtype=torch.bfloat16)
    x2, w2 = torch.zeros((M, 2 * K), dtype=torch.bfloat16), torch.zeros((N, 2 * K), dtype=torch.bfloat16)
    a.forward(x, w)
    b.forward(x2, w2)
    per_call = 1 if arm == "flux" else 2  # pull: one launch per call; push: producer + receiver
    assert [c[1]["epoch"] for c in fake.calls] == [e for e in (1, 2) for _ in range(per_call)]
    fake.fail_push = True
    with pytest.raises(RuntimeError, match="injected"):
        a.forward(x, w)
    fake.fail_push = False
    n = len(fake.calls)
    with pytest.raises(RuntimeError, match="previously failed"):
        b.forward(x2, w2)
    assert len(fake.calls) == n


@pytest.mark.parametrize("arm", ["flux", "flux_taco"])
def test_concurrent_calls_keep_each_epoch_together(monkeypatch, arm):
    import threading
    import time
    from tempname_5090_b200.parallel import gemm_rs

    class Yielding(_FakeLib):
        def gemm_rs_push(self, *a, **k):
            time.sleep(0)  # invite a thread switch between the two phases of one call
            super().gemm_rs_push(*a, **k)
            time.sleep(0)

        def gemm_rs_pull(self, *a, **k):
            time.sleep(0)
            super().gemm_rs_pull(*a, **k)
            time.sleep(0)
    fake = Yielding()
    monkeypatch.setattr(gemm_rs, "lib", lambda: fake)
    monkeypatch.setattr(gemm_rs, "count_launch", lambda n=1: None)
    op = gemm_rs.GemmRS(M, N, K, arm=arm, _emulate=(0, 2, [_Buf(1), _Buf(2)], _Buf(3)), device="cpu")
    x, w = torch.zeros((M, K), dtype=torch.bfloat16), torch.zeros((N, K), dtype=torch.bfloat16)
    threads = [threading.Thread(target=lambda: [op.forward(x, w) for _ in range(40)]) for _ in range(3)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    calls = fake.calls
    if arm == "flux":
        assert [c[1]["epoch"] for c in calls] == list(range(1, 121)) and op.epoch == 120
        return
    assert len(calls) == 2 * 120 and op.epoch == 120
    for i in range(0, len(calls), 2):
        assert calls[i][0] == "push" and calls[i + 1][0] == "reduce"
        assert calls[i][1]["epoch"] == calls[i + 1][1]["epoch"] == i // 2 + 1


def test_ag_gemm_failed_launch_poisons_the_operator(monkeypatch):
    from tempname_5090_b200.parallel import ag_gemm

    class Failing(_FakeAGLib):
        fail = False

        def ag_gemm(self, *a, **k):
            if self.fail:
                raise RuntimeError("injected launch failure")
            super().ag_gemm(*a, **k)
    fake = Failing()
    monkeypatch.setattr(ag_gemm, "lib", lambda: fake)
    monkeypatch.setattr(ag_gemm, "count_launch", lambda n=1: None)
    m, k, n = 512, 256, 512
    op = ag_gemm.AGGemm(m, k, _emulate=(0, 2, _AGBuf(1), _AGBuf(2)), device="cpu")
    shard, w = torch.zeros((m // 2, k), dtype=torch.bfloat16), torch.zeros((n, k), dtype=torch.bfloat16)
    op.forward(shard, w)
    fake.fail = True
    with pytest.raises(RuntimeError, match="injected"):
        op.forward(shard, w)
    assert op.calls == 1 and op.failed  # the failed call did not advance the epoch
    fake.fail = False
    with pytest.raises(RuntimeError, match="previously failed"):
        op.forward(shard, w)
    assert len(fake.calls) == 1


def test_lane_skew_diagnostic_names_the_same_tile_on_every_rank(monkeypatch):
    """profile_call: only `delay_rank` arms the bounded publication delay, on the
    first lane-0 tile of its own (rotated) production order, and every rank
    reports that same tile as (owner, local tile id)."""
    from tempname_5090_b200.parallel import gemm_rs
    fake = _FakeLib()
    monkeypatch.setattr(gemm_rs, "lib", lambda: fake)
    monkeypatch.setattr(gemm_rs, "count_launch", lambda n=1: None)
    monkeypatch.setattr(torch.cuda, "synchronize", lambda *a, **k: None)
    world = 4
    x, w = torch.zeros((M, K), dtype=torch.bfloat16), torch.zeros((N, K), dtype=torch.bfloat16)
    named = []
    for rank in range(world):
        op = gemm_rs.GemmRS(M, N, K, _emulate=(rank, world, [_Buf(1), _Buf(2)], _Buf(3)), device="cpu")
        fake.calls.clear()
        _, _, delayed = op.profile_call(x, w, delay_ns=1000, delay_rank=2)
        named.append(delayed)
        delay_tile, delay_ns = fake.calls[0][1]["delay"]
        if rank == 2:
            tiles_n = N // 256
            per_dest_m = M // world // 128
            tm = delay_tile // tiles_n
            dest = tm // per_dest_m
            assert delay_ns == 1000 and delayed == (dest, (tm - dest * per_dest_m) * tiles_n + delay_tile % tiles_n)
            assert dest == 3  # rank 2 produces for destination 3 first
        else:
            assert (delay_tile, delay_ns) == (-1, 0)
    assert len(set(named)) == 1


def test_device_failure_poisons_every_live_fused_operator(monkeypatch):
    """A bounded-wait failure reported by the device poisons every live fused
    operator and exchange workspace: none of them launches again."""
    from tempname_5090_b200 import _native
    from tempname_5090_b200.parallel import gemm_rs, ag_gemm
    fake, fake_ag = _FakeLib(), _FakeAGLib()
    monkeypatch.setattr(gemm_rs, "lib", lambda: fake)
    monkeypatch.setattr(gemm_rs, "count_launch", lambda n=1: None)
    monkeypatch.setattr(ag_gemm, "lib", lambda: fake_ag)
    monkeypatch.setattr(ag_gemm, "count_launch", lambda n=1: None)
    rs = gemm_rs.GemmRS(M, N, K, _emulate=(0, 2, [_Buf(1), _Buf(2)], _Buf(3)), device="cpu")
    ag = ag_gemm.AGGemm(512, 256, _emulate=(0, 2, _AGBuf(4), _AGBuf(5)), device="cpu")
    x, w = torch.zeros((M, K), dtype=torch.bfloat16), torch.zeros((N, K), dtype=torch.bfloat16)
    rs.forward(x, w)
    assert _native.poison_operators() >= 3  # the operator, its workspace and the AG operator
    assert rs.failed and rs.workspace.failed and ag.failed
    with pytest.raises(RuntimeError, match="previously failed"):
        rs.forward(x, w)
    with pytest.raises(RuntimeError, match="previously failed"):
        ag.forward(torch.zeros((256, 256), dtype=torch.bfloat16), torch.zeros((512, 256), dtype=torch.bfloat16))
    assert len(fake.calls) == 1 and fake_ag.calls == []
