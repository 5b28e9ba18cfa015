"""Fused GEMM->RS and AG->GEMM kernels with W ranks emulated on ONE GPU.

Every rank's buffers are local allocations; each emulated rank's kernels are
launched in an order where every wait is already satisfied when the kernel
starts (producers before receivers, peers' pushes pre-filled), so no launch
ever waits on another launch.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _gen(seed):
    return torch.Generator(device="cuda").manual_seed(seed)


@pytest.mark.parametrize("world,blocks", [(2, 2), (4, 2), (8, 2), (2, 3), (8, 3)])
@pytest.mark.parametrize("arm", ["flux", "flux_taco", "flux_taco_interleaved", "flux_taco_interleaved_arrival"])
def test_gemm_rs_emulated_bitwise(world, blocks, arm):
    """Every arm against an ordered reduce / decode_reduce of the partials.
    An odd block count per destination leaves lane 1 one block shorter than
    lane 0 (push transport)."""
    from tempname_5090_b200.parallel.gemm_rs import GemmRS
    from tempname_5090_b200.parallel.symmetric import SymmetricBuffer
    from tempname_5090_b200.parallel import planning, mapping
    from tempname_5090_b200.ops import gemm as G, taco
    from tempname_5090_b200._native import check_status
    chunk = 128
    m, n, k = world * blocks * chunk, 512, 320
    rows = m // world
    lanes = mapping.PushLanes(rows, n, chunk, world)
    recv = [SymmetricBuffer.emulated(lanes.recv_bytes, world) for _ in range(2)]
    flags = SymmetricBuffer.emulated(max(lanes.flag_words, world * (rows // 128) * (n // 256)) * 4, world)
    plan = None
    if arm.endswith("arrival"):
        order = planning.candidates(m, n, k, world, chunk)[1]["arrival_order"]
        plan = planning.make_role(m, n, k, world, chunk, order)
    ops = [GemmRS(m, n, k, arm=arm, chunk_rows=chunk, plan=plan,
                  _emulate=(r, world, [b.as_rank(r) for b in recv], flags.as_rank(r))) for r in range(world)]
    xs = [torch.randn((m, k), generator=_gen(r), device="cuda").to(torch.bfloat16) for r in range(world)]
    ws = [(0.05 * torch.randn((n, k), generator=_gen(100 + r), device="cuda")).to(torch.bfloat16) for r in range(world)]
    for call in range(3):  # several calls exercise both slot parities and epochs
        for op in ops:
            op.begin()
        for r, op in enumerate(ops):
            op.push(xs[r], ws[r])
        outs = []
        for op in ops:
            out = torch.empty((rows, n), dtype=torch.bfloat16, device="cuda")
            op.reduce(out)
            outs.append(out)
        torch.cuda.synchronize()
        check_status()
        partials = [G.matmul(xs[s], ws[s], bn=256) for s in range(world)]
        for r in range(world):
            local = partials[r][r * rows:(r + 1) * rows].contiguous()
            if op.quantized:
                blocks = []
                for b in range(rows // chunk):
                    pk = [taco.encode(partials[s][r * rows + b * chunk: r * rows + (b + 1) * chunk])
                          for s in range(world) if s != r]
                    blocks.append(taco.decode_reduce(local[b * chunk:(b + 1) * chunk].contiguous(),
                                                     torch.cat(pk), r, world))
                expect = torch.cat(blocks)
            else:
                remote = torch.cat([partials[s][r * rows:(r + 1) * rows] for s in range(world) if s != r])
                expect = taco.ordered_reduce(local, remote, r, world)
            assert torch.equal(outs[r], expect), (arm, world, r, call)
        xs = [(x * 0.5 + 0.25).to(torch.bfloat16) for x in xs]


@pytest.mark.parametrize("blocks", [2, 3])
def test_push_lanes_have_their_own_regions_and_flags(blocks):
    """Push transport, W=2 emulated, BF16 arm: after both producers ran (no
    receiver yet), each owner's lane l holds exactly the rows of its blocks
    2j + l from each source (lane region [source][lane block]) and that lane's
    flag array has the epoch at the lane's tiles; padding of a shorter lane
    stays untouched."""
    from tempname_5090_b200.parallel.gemm_rs import GemmRS
    from tempname_5090_b200.parallel.symmetric import SymmetricBuffer
    from tempname_5090_b200.parallel.mapping import PushLanes
    from tempname_5090_b200.ops import gemm as G
    from tempname_5090_b200._native import check_status
    world, chunk, n, k = 2, 128, 512, 192
    m = world * blocks * chunk
    rows = m // world
    lanes = PushLanes(rows, n, chunk, world)
    recv = [SymmetricBuffer.emulated(lanes.recv_bytes, world) for _ in range(2)]
    flags = SymmetricBuffer.emulated(lanes.flag_words * 4, world)
    ops = [GemmRS(m, n, k, arm="flux", pull=False, chunk_rows=chunk,
                  _emulate=(r, world, [b.as_rank(r) for b in recv], flags.as_rank(r))) for r in range(world)]
    xs = [torch.randn((m, k), generator=_gen(30 + r), device="cuda").to(torch.bfloat16) for r in range(world)]
    ws = [torch.randn((n, k), generator=_gen(40 + r), device="cuda").to(torch.bfloat16) for r in range(world)]
    for op in ops:
        op.begin()
    for r, op in enumerate(ops):
        op.push(xs[r], ws[r])
    torch.cuda.synchronize()
    check_status()
    parts = [G.matmul(xs[s], ws[s], bn=256) for s in range(world)]
    parity = ops[0].epoch & 1
    for r in range(world):
        region = recv[parity].as_rank(r).local_view((lanes.recv_bytes // 2,), torch.bfloat16)
        words = flags.as_rank(r).local_view((lanes.flag_words,), torch.int32)
        expect_flags = torch.zeros_like(words)
        expect_flags[torch.tensor(lanes.flag_indices(), device=words.device)] = ops[r].epoch
        assert torch.equal(words, expect_flags), (blocks, r)
        for lane in range(2):
            for s in range(world):
                off = lanes.slot_offset(lane, s)
                slot = region[off // 2: off // 2 + lanes.lane_slot_bytes // 2].view(-1, n)
                for j, b in enumerate(range(lane, blocks, 2)):
                    got = slot[j * chunk:(j + 1) * chunk]
                    want = parts[s][r * rows + b * chunk: r * rows + (b + 1) * chunk]
                    assert torch.equal(got, want), (blocks, r, lane, s, b)


def test_gemm_rs_fused_residual_bias():
    from tempname_5090_b200.parallel.gemm_rs import GemmRS
    from tempname_5090_b200.parallel.symmetric import SymmetricBuffer
    from tempname_5090_b200.ops import gemm as G, taco
    from tempname_5090_b200.parallel.mapping import PushLanes
    world, m, n, k = 2, 512, 256, 128
    rows = m // world
    lanes = PushLanes(rows, n, 128, world)
    recv = [SymmetricBuffer.emulated(lanes.recv_bytes, world) for _ in range(2)]
    flags = SymmetricBuffer.emulated(lanes.flag_words * 4, world)
    ops = [GemmRS(m, n, k, _emulate=(r, world, [b.as_rank(r) for b in recv], flags.as_rank(r))) for r in range(world)]
    xs = [torch.randn((m, k), generator=_gen(r), device="cuda").to(torch.bfloat16) for r in range(world)]
    ws = [torch.randn((n, k), generator=_gen(9 + r), device="cuda").to(torch.bfloat16) for r in range(world)]
    res = torch.randn((rows, n), generator=_gen(5), device="cuda").to(torch.bfloat16)
    bias = torch.randn((n,), generator=_gen(6), device="cuda").to(torch.bfloat16)
    for op in ops:
        op.begin()
    for r, op in enumerate(ops):
        op.push(xs[r], ws[r])
    out = torch.empty((rows, n), dtype=torch.bfloat16, device="cuda")
    ops[0].reduce(out, residual=res, bias=bias)
    plain = torch.empty_like(out)
    ops[1].reduce(torch.empty_like(out))
    parts = [G.matmul(xs[s], ws[s], bn=256) for s in range(world)]
    y = taco.ordered_reduce(parts[0][:rows].contiguous(), parts[1][:rows].contiguous(), 0, world)
    expect = ((res.float() + y.float()).to(torch.bfloat16).float() + bias.float()).to(torch.bfloat16)
    assert torch.equal(out, expect)


@pytest.mark.parametrize("world,bn,kind", [(2, 128, 0), (4, 256, 0), (8, 256, 0), (2, 256, 2), (8, 256, 2)])
@pytest.mark.parametrize("epi", ["plain", "bias_gelu", "mn_major", "in_place"])
def test_ag_gemm_emulated(world, bn, kind, epi):
    """Pull all-gather -> GEMM, W ranks emulated on one GPU: every rank's call
    runs as three launches (own chunk + publish, pull peers, GEMM) over all ranks
    in turn.  Three calls with changing inputs exercise the cumulative counters
    and the `pulled` handshake that guards the own chunk between calls."""
    from tempname_5090_b200.parallel.ag_gemm import AGGemm, control_layout
    from tempname_5090_b200.parallel.symmetric import SymmetricBuffer
    from tempname_5090_b200.ops import gemm as G
    from tempname_5090_b200._native import check_status
    m, k, n = world * 256, 320, (1024 if kind else 768)
    rows = m // world
    gather = SymmetricBuffer.emulated(m * k * 2, world)
    pulled_offset, ctrl_bytes = control_layout(m)
    ctrl = SymmetricBuffer.emulated(ctrl_bytes, world)
    ops = [AGGemm(m, k, comm_ctas=4 if kind else 3, tile_kind=kind,
                  _emulate=(r, world, gather.as_rank(r), ctrl.as_rank(r))) for r in range(world)]
    w = (0.05 * torch.randn((n, k), generator=_gen(77), device="cuda")).to(torch.bfloat16)
    w_mn = w.t().contiguous()
    bias = torch.randn((n,), generator=_gen(78), device="cuda").to(torch.bfloat16)
    for call in range(3):
        shards = [torch.randn((rows, k), generator=_gen(10 * call + r), device="cuda").to(torch.bfloat16)
                  for r in range(world)]
        full = torch.cat(shards)
        weight = w_mn if epi == "mn_major" else w
        kw = dict(b_mn=epi == "mn_major", bn=bn)
        if epi == "bias_gelu":
            kw["bias"] = bias
        if epi == "in_place":
            # the shard is written straight into the own chunk (after the bounded
            # wait input_buffer launches) and published without a copy
            views = [ops[r].input_buffer() for r in range(world)]
            for r in range(world):
                views[r].copy_(shards[r])
            shards = views
        for phase in (1, 2):
            for r in range(world):
                ops[r].forward(shards[r], weight, phase=phase, **kw)
        outs, auxs = [], []
        for r in range(world):
            aux = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
            extra = dict(gelu_aux=aux) if epi == "bias_gelu" else {}
            outs.append(ops[r].forward(shards[r], weight, phase=4, **kw, **extra))
            auxs.append(aux)
        torch.cuda.synchronize()
        check_status()
        aux_ref = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
        extra = dict(gelu_aux=aux_ref) if epi == "bias_gelu" else {}
        expect = G.matmul(full, weight, b_t=epi == "mn_major", bias=kw.get("bias"), bn=bn, pair=kind, **extra)
        for r in range(world):
            assert torch.equal(ops[r].gathered, full), (r, call)
            assert torch.equal(outs[r], expect), (r, call)
            if epi == "bias_gelu":
                assert torch.equal(auxs[r], aux_ref)
        # every peer signalled once per gatherer CTA per call
        pulled = [int(ctrl.view(r, (ctrl_bytes // 4,), torch.int32)[pulled_offset // 4].item()) for r in range(world)]
        assert pulled == [(world - 1) * ops[0].comm_ctas * (call + 1)] * world, pulled


@pytest.mark.parametrize("world", [2, 8])
@pytest.mark.parametrize("comm_ctas,kind", [(1, 0), (5, 0), (20, 0), (4, 2), (16, 2)])
def test_gemm_rs_pull_emulated_matches_push(world, comm_ctas, kind):
    """Pull transport (GEMM launch, then reducer launch, per emulated rank) is
    bitwise equal to the push transport and to the ordered reduce of the
    partials, with residual + bias, over calls of both buffer parities."""
    from tempname_5090_b200.parallel.gemm_rs import GemmRS
    from tempname_5090_b200.parallel.symmetric import SymmetricBuffer
    from tempname_5090_b200.ops import gemm as G, taco
    from tempname_5090_b200._native import check_status
    m, n, k = (world * 512, 1024, 640) if kind else (world * 384, 768, 448)
    rows = m // world
    tiles = (rows // 128) * (n // 256)
    bufs = {}
    ops = {}
    for pull in (True, False):
        data = [SymmetricBuffer.emulated(m * n * 2, world) for _ in range(2)]
        flags = SymmetricBuffer.emulated(world * tiles * 4, world)
        bufs[pull] = data + [flags]
        ops[pull] = [GemmRS(m, n, k, pull=pull, comm_ctas=comm_ctas, tile_kind=kind if pull else None,
                            _emulate=(r, world, [b.as_rank(r) for b in data], flags.as_rank(r)))
                     for r in range(world)]
    res = torch.randn((rows, n), generator=_gen(5), device="cuda").to(torch.bfloat16)
    bias = torch.randn((n,), generator=_gen(6), device="cuda").to(torch.bfloat16)
    for call in range(3):
        xs = [torch.randn((m, k), generator=_gen(40 * call + r), device="cuda").to(torch.bfloat16)
              for r in range(world)]
        ws = [(0.05 * torch.randn((n, k), generator=_gen(200 + r), device="cuda")).to(torch.bfloat16)
              for r in range(world)]
        outs = {}
        for pull, group in ops.items():
            for op in group:
                op.begin()
            for r, op in enumerate(group):
                op.push(xs[r], ws[r])
            outs[pull] = []
            for r, op in enumerate(group):
                out = torch.empty((rows, n), dtype=torch.bfloat16, device="cuda")
                op.reduce(out, residual=res if call else None, bias=bias if call else None)
                outs[pull].append(out)
        torch.cuda.synchronize()
        check_status()
        # partials of the pull GEMM's own tile kind (the push transport uses single-CTA tiles)
        partials = [G.matmul(xs[s], ws[s], bn=256, pair=kind) for s in range(world)]
        for r in range(world):
            local = partials[r][r * rows:(r + 1) * rows].contiguous()
            remote = torch.cat([partials[s][r * rows:(r + 1) * rows] for s in range(world) if s != r])
            y = taco.ordered_reduce(local, remote, r, world)
            if call:
                y = ((res.float() + y.float()).to(torch.bfloat16).float() + bias.float()).to(torch.bfloat16)
            assert torch.equal(outs[True][r], y), (world, comm_ctas, call, r)
            if kind == 0:
                assert torch.equal(outs[True][r], outs[False][r])
            else:
                ref = outs[False][r].float()
                assert ((outs[True][r].float() - ref).norm() / ref.norm()).item() < 1e-2
    for group in bufs.values():
        for b in group:
            b.close()


def test_gemm_rs_pull_signed_zero_and_order():
    """The BF16 adds of the pull reducer keep the reference's rounding and
    signed-zero behaviour: sources holding -0.0 and values that cancel or round
    differently in another order."""
    from tempname_5090_b200.parallel.gemm_rs import GemmRS
    from tempname_5090_b200.parallel.symmetric import SymmetricBuffer
    from tempname_5090_b200.ops import taco
    from tempname_5090_b200._native import check_status
    world, m, n, k = 4, 512, 256, 64
    rows = m // world
    data = [SymmetricBuffer.emulated(m * n * 2, world) for _ in range(2)]
    flags = SymmetricBuffer.emulated(world * (rows // 128) * (n // 256) * 4, world)
    ops = [GemmRS(m, n, k, pull=True, comm_ctas=2, _emulate=(r, world, [b.as_rank(r) for b in data], flags.as_rank(r)))
           for r in range(world)]
    # x = e_0 (one-hot K) so each partial row equals a chosen weight column: partial[r, c] = w[c, 0]
    vals = [torch.tensor([-0.0, 1.0, 2.0 ** -9, -1.0], dtype=torch.float32),
            torch.tensor([-0.0, 2.0 ** -9, 2.0 ** -9, 1.0], dtype=torch.float32),
            torch.tensor([-0.0, 2.0 ** -9, -1.0, 3.0e38], dtype=torch.float32),
            torch.tensor([-0.0, -1.0, 1.0, -3.0e38], dtype=torch.float32)]
    x = torch.zeros((m, k), dtype=torch.bfloat16, device="cuda")
    x[:, 0] = 1
    ws = []
    for s in range(world):
        w = torch.zeros((n, k), dtype=torch.float32)
        w[:, 0] = vals[s].repeat(n // 4)
        ws.append(w.to(torch.bfloat16).cuda())
    for op in ops:
        op.begin()
    for r, op in enumerate(ops):
        op.push(x, ws[r])
    outs = []
    for op in ops:
        out = torch.empty((rows, n), dtype=torch.bfloat16, device="cuda")
        op.reduce(out)
        outs.append(out)
    torch.cuda.synchronize()
    check_status()
    from tempname_5090_b200.ops import gemm as G
    parts = [G.matmul(x, ws[s], bn=256) for s in range(world)]  # the same tile kind as the fused GEMM
    for r in range(world):
        expect = taco.ordered_sum_cpu([p[r * rows:(r + 1) * rows].cpu() for p in parts])
        got = outs[r].cpu()
        assert torch.equal(got.view(torch.int16), expect.view(torch.int16)), r


def test_bounded_wait_times_out_and_context_survives():
    from tempname_5090_b200._native import lib, status_tensor, check_status
    flag = torch.zeros(4, dtype=torch.int32, device="cuda")
    status = status_tensor("cuda")
    status.zero_()
    lib().wait_probe(flag.data_ptr(), 1, 200_000_000, status)  # 0.2 s, nothing ever sets it
    torch.cuda.synchronize()
    assert int(status[0].item()) == 5
    status.zero_()
    x = torch.ones(8, device="cuda")
    assert x.sum().item() == 8.0  # context still usable
    check_status()


@pytest.mark.parametrize("arm", ["flux", "flux_taco"])
def test_guard_regions_stay_intact_and_detect_an_overrun(arm):
    """Guarded receive slots and flags around emulated GemmRS calls: every
    rank's guards keep their pattern; a byte written into a guard (on purpose,
    from the host side) is reported for that rank."""
    from tempname_5090_b200.parallel.gemm_rs import GemmRS
    from tempname_5090_b200.parallel.symmetric import SymmetricBuffer
    from tempname_5090_b200._native import check_status, lib
    from tempname_5090_b200.parallel.mapping import PushLanes
    world, m, n, k = 4, 1024, 512, 256
    rows = m // world
    g = 4096
    lanes = PushLanes(rows, n, 128, world)
    recv = [SymmetricBuffer(lanes.recv_bytes, guard_bytes=g, _emulate_world=world) for _ in range(2)]
    flags = SymmetricBuffer(lanes.flag_words * 4, guard_bytes=g, _emulate_world=world)
    ops = [GemmRS(m, n, k, arm=arm, _emulate=(r, world, [b.as_rank(r) for b in recv], flags.as_rank(r)))
           for r in range(world)]
    xs = [torch.randn((m, k), generator=_gen(r), device="cuda").to(torch.bfloat16) for r in range(world)]
    ws = [(0.05 * torch.randn((n, k), generator=_gen(50 + r), device="cuda")).to(torch.bfloat16) for r in range(world)]
    for _ in range(3):
        for op in ops:
            op.begin()
        for r, op in enumerate(ops):
            op.push(xs[r], ws[r])
        for op in ops:
            op.reduce(torch.empty((rows, n), dtype=torch.bfloat16, device="cuda"))
    torch.cuda.synchronize()
    check_status()
    assert all(b.check_guards() == [] for b in recv + [flags])
    # Corrupt the trailing guard of rank 2's flag region and the leading guard of rank 1's slot 0.
    lib().view_ptr(flags.peers[2] + flags.nbytes + 7, [1], torch.uint8, 0).fill_(0)
    lib().view_ptr(recv[0].peers[1] - 1, [1], torch.uint8, 0).fill_(0)
    assert flags.check_guards() == [2]
    assert recv[0].check_guards() == [1]
    assert recv[1].check_guards() == []
    for b in recv + [flags]:
        b.close()


@pytest.mark.parametrize("arm,kind", [("flux", 0), ("flux", 2), ("flux_taco", 0), ("flux_taco_interleaved", 0)])
def test_mapping_probe_reads_back_the_host_production_order(arm, kind):
    """The device decodes each operator's uploaded production table into
    exactly the host's tile order (every tile once, the rotated / interleaved
    destination sequence) -- the mapping probe of the validation gate."""
    from tempname_5090_b200.parallel.gemm_rs import GemmRS
    from tempname_5090_b200.parallel.symmetric import SymmetricBuffer
    world, m, n, k = 4, 2048, 1024, 512
    data = [SymmetricBuffer.emulated(m * n * 2, world) for _ in range(2)]
    flags = SymmetricBuffer.emulated(world * (m // world // 128) * (n // 256) * 4, world)
    for r in range(world):
        op = GemmRS(m, n, k, arm=arm, tile_kind=kind if arm == "flux" else None,
                    _emulate=(r, world, [b.as_rank(r) for b in data], flags.as_rank(r)))
        host = op.host_tile_map()
        assert op.device_tile_map() == host
        assert len(set(host)) == len(host) == (m // op.tile_m) * (n // op.tile_n)
    for b in data + [flags]:
        b.close()


@pytest.mark.parametrize("world", [2, 8])
def test_pull_scatter_of_an_existing_tensor(world):
    """The embedding's SumScatter over the pull transport (pack, publish,
    reducer-only launch): bitwise the ordered BF16 sum of the sources' rows,
    over calls of both buffer parities."""
    from tempname_5090_b200.parallel.gemm_rs import GemmRS
    from tempname_5090_b200.parallel.symmetric import SymmetricBuffer
    from tempname_5090_b200.ops import taco
    from tempname_5090_b200._native import check_status
    m, n = world * 256, 768
    rows = m // world
    data = [SymmetricBuffer.emulated(m * n * 2, world) for _ in range(2)]
    flags = SymmetricBuffer.emulated(world * (rows // 128) * (n // 256) * 4, world)
    ops = [GemmRS(m, n, 8, comm_ctas=6, _emulate=(r, world, [b.as_rank(r) for b in data], flags.as_rank(r)))
           for r in range(world)]
    for call in range(3):
        xs = [torch.randn((m, n), generator=_gen(9 * call + r), device="cuda").to(torch.bfloat16)
              for r in range(world)]
        if call == 1:  # embedding-like: each row non-zero on exactly one source
            owner = torch.randint(0, world, (m,), generator=torch.Generator().manual_seed(5))
            xs = [x * (owner == r).to(x.device)[:, None].to(torch.bfloat16) for r, x in enumerate(xs)]
        for r, op in enumerate(ops):
            op.scatter(xs[r], phase=1)
        outs = [op.scatter(xs[r], phase=2) for r, op in enumerate(ops)]
        torch.cuda.synchronize()
        check_status()
        for r in range(world):
            local = xs[r][r * rows:(r + 1) * rows].contiguous()
            remote = torch.cat([xs[s][r * rows:(r + 1) * rows] for s in range(world) if s != r])
            assert torch.equal(outs[r], taco.ordered_reduce(local, remote, r, world)), (call, r)
            if call == 1:
                assert torch.equal(outs[r], sum(x.float() for x in xs)[r * rows:(r + 1) * rows].to(torch.bfloat16))
    for b in data + [flags]:
        b.close()
