"""Expert parallelism with the fused CUDA FFN: one GPU in-process, two GPUs (NCCL) when visible."""

from __future__ import annotations

import os
import socket

import pytest
import torch

from oracle import moe_ffn as O

pytestmark = pytest.mark.gpu

E, H, I, T, K = 8, 256, 128, 300, 4


def _check_ep(tag, got, want, rank, e_local):
    """got: this rank's (out, dx, dw_router, dw_up, db_up, dw_down, db_down); want: ep_reference()."""
    sl = slice(rank * e_local, (rank + 1) * e_local)
    pairs = [("out", got[0], want["out"][rank]), ("dx", got[1], want["dx"][rank]),
             ("dw_router", got[2], want["dw_router"][rank]), ("dw_up", got[3], want["dw_up"][sl]),
             ("db_up", got[4], want["db_up"][sl]), ("dw_down", got[5], want["dw_down"][sl]),
             ("db_down", got[6], want["db_down"][sl])]
    for name, a, b in pairs:
        r = O.check(f"{tag}:rank{rank}:{name}", torch.as_tensor(a).float(), b.float())
        assert r["ok"], r


def test_ep_world1_matches_oracle():
    """One rank: outputs, token and router-weight gradients and all four weight/bias gradients
    against the single-process oracle, with router weights and a random output gradient."""
    from cutlass_op.bf16_grouped_mm.expert_parallel import EPMoEFFN, route_tokens
    from oracle.ep_ffn import ep_reference

    dev = torch.device("cuda", 0)
    ffn = EPMoEFFN(E, H, I, device=dev, seed=5)
    g = torch.Generator().manual_seed(1)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    w = torch.rand(T, K, generator=g)
    gout = torch.randn(T, H, generator=g).to(torch.bfloat16)
    idx = route_tokens(T, E, K, "zipf", seed=2)
    xd = x.to(dev).requires_grad_(True)
    wd = w.to(dev).requires_grad_(True)
    out = ffn(xd, idx.to(dev), wd)
    out.backward(gout.to(dev))
    torch.cuda.synchronize()
    want = ep_reference([x], [idx], [w], [gout], *[p.detach().cpu() for p in
                                                    (ffn.w_up, ffn.b_up, ffn.w_down, ffn.b_down)])
    got = [t.detach().cpu() for t in (out, xd.grad, wd.grad, ffn.w_up.grad, ffn.b_up.grad, ffn.w_down.grad,
                                      ffn.b_down.grad)]
    _check_ep("world1", got, want, 0, E)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_row_kernels_match_torch():
    """gather_rows / combine_rows against torch indexing, with and without scales."""
    g = torch.Generator().manual_seed(3)
    src = torch.randn(50, 264, generator=g).to(torch.bfloat16).cuda()
    idx = torch.randint(0, 50, (77,), generator=g).cuda()
    sc = torch.rand(77, generator=g).cuda()
    assert torch.equal(torch.ops.grouped_mm.gather_rows(src, idx, None), src[idx])
    ref = (src[idx].float() * sc.unsqueeze(1)).to(torch.bfloat16)
    assert torch.allclose(torch.ops.grouped_mm.gather_rows(src, idx, sc).float(), ref.float(), rtol=1e-2, atol=1e-2)
    k = 3
    pos = torch.randint(0, 50, (20 * k,), generator=g).cuda()
    w = torch.rand(20 * k, generator=g).cuda()
    out = torch.ops.grouped_mm.combine_rows(src, pos, w, k)
    ref = (src[pos].float() * w.unsqueeze(1)).view(20, k, -1).sum(1)
    r = O.check("combine", out.float().cpu(), ref.cpu())
    assert r["ok"], r


def test_row_kernels_flag_out_of_range_index():
    """An index outside the source rows is skipped, its output row keeps its old contents, the
    other rows are right, and MGF_DEV_ROW_OUT_OF_RANGE is recorded (read and cleared)."""
    import ctypes

    from cutlass_op.bf16_grouped_mm import _ext

    lib = _ext.lib
    _ext.device_status(clear=True)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    g = torch.Generator().manual_seed(11)
    src = torch.randn(40, 64, generator=g).to(torch.bfloat16).cuda()
    idx = torch.tensor([3, 39, 40, 0, -1, 7], dtype=torch.int64).cuda()   # 40 and -1 are outside
    dst = torch.full((6, 64), 5.0, dtype=torch.bfloat16).cuda()
    rc = lib.mgf_gather_rows(ctypes.c_void_p(src.data_ptr()), ctypes.c_int64(64), ctypes.c_int64(40),
                             ctypes.c_void_p(idx.data_ptr()), None, ctypes.c_int64(6), ctypes.c_int64(64),
                             ctypes.c_void_p(dst.data_ptr()), ctypes.c_int64(64), stream)
    assert rc == 0
    torch.cuda.synchronize()
    good = [0, 1, 3, 5]
    assert torch.equal(dst[good], src[idx[good]])
    assert (dst[[2, 4]].float() == 5.0).all()
    assert _ext.device_status(clear=True) == _ext.DEV_ROW_OUT_OF_RANGE
    # combine: a token with one bad slot is left untouched, the others are summed
    k = 2
    pos = torch.tensor([0, 1, 2, 99, 4, 5], dtype=torch.int64).cuda()
    out = torch.full((3, 64), 5.0, dtype=torch.bfloat16).cuda()
    rc = lib.mgf_combine_rows(ctypes.c_void_p(src.data_ptr()), ctypes.c_int64(64), ctypes.c_int64(40),
                              ctypes.c_void_p(pos.data_ptr()), None, ctypes.c_int64(3), ctypes.c_int32(k),
                              ctypes.c_int64(64), ctypes.c_void_p(out.data_ptr()), ctypes.c_int64(64), stream)
    assert rc == 0
    torch.cuda.synchronize()
    ref = (src[[0, 4]].float() + src[[1, 5]].float()).to(torch.bfloat16)
    assert torch.equal(out[[0, 2]], ref)
    assert (out[1].float() == 5.0).all()
    assert _ext.device_status(clear=True) == _ext.DEV_ROW_OUT_OF_RANGE
    with pytest.raises(RuntimeError, match="outside its buffer"):
        torch.ops.grouped_mm.gather_rows(src, idx, None)
        _ext.check_device_status()
    assert _ext.device_status(clear=True) == 0


def test_ep_autograd_row_functions():
    """Gradients of dispatch / permute / combine through the kernels equal torch autograd's."""
    from cutlass_op.bf16_grouped_mm.expert_parallel import DispatchPlan, _Combine, _Dispatch, route_tokens

    idx = route_tokens(40, 6, 3, "zipf", seed=9).cuda()
    plan = DispatchPlan(idx, 6, 1)
    x = torch.randn(40, 64, generator=torch.Generator().manual_seed(4)).to(torch.bfloat16).cuda().requires_grad_(True)
    w = torch.rand(40, 3, generator=torch.Generator().manual_seed(5)).cuda().requires_grad_(True)
    send = _Dispatch.apply(x, plan.copy_token, plan.inv_order, 3)
    y = send * 2
    out = _Combine.apply(y, plan.inv_order, plan.copy_token, plan.order, w.reshape(-1), 3)
    go = torch.randn(40, 64, generator=torch.Generator().manual_seed(6)).to(torch.bfloat16).cuda()
    out.backward(go)
    x2 = x.detach().float().requires_grad_(True)
    w2 = w.detach().requires_grad_(True)
    ref = (2 * x2.unsqueeze(1) * w2.unsqueeze(2)).sum(1)
    ref.backward(go.float())
    for name, a, b in (("out", out, ref), ("dx", x.grad, x2.grad), ("dw", w.grad, w2.grad)):
        r = O.check(name, a.float().cpu(), b.detach().cpu())
        assert r["ok"], r


def _transport_worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        from conftest import PKG  # noqa: F401

        import torch.distributed as dist

        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
        try:
            from cutlass_op.bf16_grouped_mm.expert_parallel import EPMoEFFN, route_tokens

            res = {}
            gen = torch.Generator().manual_seed(10 + rank)
            x0 = torch.randn(T, H, generator=gen).to(torch.bfloat16)
            w0 = torch.rand(T, K, generator=gen)
            g0 = torch.randn(T, H, generator=gen).to(torch.bfloat16)
            idx = route_tokens(T, E, K, "zipf", seed=20 + rank)
            res["inputs"] = [x0.float().numpy(), idx.numpy(), w0.numpy(), g0.float().numpy()]
            for transport in ("nccl", "peer", "peer_pipeline", "peer_unfused", "peer_overlap"):
                ffn = EPMoEFFN(E, H, I, device=dev, seed=5, transport=transport.split("_")[0],
                               overlap=transport.endswith("overlap"), fused=transport in ("peer", "peer_pipeline"),
                               pipeline=transport == "peer_pipeline")
                x = x0.to(dev).requires_grad_(True)
                w = w0.to(dev).requires_grad_(True)
                for step in range(2):  # the second step reuses the peer buffers
                    x.grad = None
                    w.grad = None
                    ffn.zero_grad()
                    out = ffn(x, idx.to(dev), w)
                    out.backward(g0.to(dev))
                torch.cuda.synchronize()
                res[transport] = [t.detach().float().cpu().numpy() for t in
                                  (out, x.grad, w.grad, ffn.w_up.grad, ffn.b_up.grad, ffn.w_down.grad,
                                   ffn.b_down.grad)]
            # every rank's expert weights, so the parent can build the single-process oracle
            gathered = []
            for p in (ffn.w_up, ffn.b_up, ffn.w_down, ffn.b_down):
                parts = [torch.empty_like(p) for _ in range(world)]
                dist.all_gather(parts, p.detach().contiguous())
                gathered.append(torch.cat(parts, 0).float().cpu().numpy())
            res["weights"] = gathered
            q.put((rank, res))
        finally:
            dist.destroy_process_group()
    except Exception:
        import traceback

        q.put((rank, "error", traceback.format_exc()))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_world2_every_transport_matches_oracle():
    """Two ranks, Zipf routing, router weights, a random output gradient, two steps: for the NCCL
    all-to-all, the peer transport with the combine / dispatch gradient fused into the GEMM epilogues
    (the default), the peer transport with separate pushes, and that with the overlapped dispatch
    gradient, each rank's output, token gradient, router-weight gradient and its experts' weight and
    bias gradients match the single-process oracle over both ranks' tokens; the overlap changes no
    bit, and the fused epilogues give the separate pushes' results bit for bit."""
    import torch.multiprocessing as mp

    from oracle.ep_ffn import ep_reference

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_transport_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(2):
            r = q.get(timeout=300)
            assert not (isinstance(r[1], str) and r[1] == "error"), r[2]
            res[r[0]] = r[1]
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for p in procs:
        assert p.exitcode == 0
    bf = torch.bfloat16
    ins = [res[r]["inputs"] for r in range(2)]
    wts = [torch.from_numpy(a).to(bf) for a in res[0]["weights"]]
    want = ep_reference([torch.from_numpy(i[0]).to(bf) for i in ins], [torch.from_numpy(i[1]) for i in ins],
                        [torch.from_numpy(i[2]) for i in ins], [torch.from_numpy(i[3]).to(bf) for i in ins], *wts)
    for rank in range(2):
        for transport in ("nccl", "peer", "peer_pipeline", "peer_unfused", "peer_overlap"):
            _check_ep(transport, [torch.from_numpy(a) for a in res[rank][transport]], want, rank, E // 2)
        for a, b in zip(res[rank]["peer_overlap"], res[rank]["peer_unfused"]):
            assert (a == b).all(), f"rank{rank}: overlap changed the result"
        for a, b in zip(res[rank]["peer"], res[rank]["peer_unfused"]):
            assert (a == b).all(), f"rank{rank}: the fused epilogues changed the result"
        for a, b in zip(res[rank]["peer_pipeline"], res[rank]["peer"]):
            assert (a == b).all(), f"rank{rank}: the pipelined halves changed the result"


def _overflow_worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        from conftest import PKG  # noqa: F401

        import torch.distributed as dist

        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
        try:
            from cutlass_op.bf16_grouped_mm import _ext
            from cutlass_op.bf16_grouped_mm.expert_parallel import EPMoEFFN, route_tokens

            _ext.device_status(clear=True)
            ffn = EPMoEFFN(E, H, I, device=dev, seed=5, capacity_factor=0.25)  # far below the ~1x received
            x = torch.randn(T, H, generator=torch.Generator().manual_seed(10 + rank)).to(torch.bfloat16)
            x = x.to(dev).requires_grad_(True)
            idx = route_tokens(T, E, K, "zipf", seed=20 + rank).to(dev)
            out = ffn(x, idx)
            out.float().sum().backward()
            torch.cuda.synchronize()
            st = _ext.device_status(clear=False)
            try:
                _ext.check_device_status()
                raised = False
            except RuntimeError:
                raised = True
            q.put((rank, {"status": st, "raised": raised, "after": _ext.device_status(clear=True)}))
        finally:
            dist.destroy_process_group()
    except Exception:
        import traceback

        q.put((rank, "error", traceback.format_exc()))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_world2_capacity_overflow_is_reported():
    """Receive buffers far below the rows a rank receives: the pushes skip the rows past the
    capacity, nothing outside the buffers is touched, and the device status word reports it on the
    host (check_device_status raises RuntimeError)."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_overflow_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(2):
            r = q.get(timeout=300)
            assert not (isinstance(r[1], str) and r[1] == "error"), r[2]
            res[r[0]] = r[1]
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for rank in range(2):
        assert res[rank]["status"] & 0x4, res[rank]        # MGF_DEV_ROW_OUT_OF_RANGE
        assert res[rank]["raised"] and res[rank]["after"] == 0, res[rank]


@pytest.mark.parametrize("world,E,T,K", [(1, 8, 300, 4), (2, 16, 517, 4), (4, 128, 1000, 4), (8, 256, 333, 8)])
def test_device_plan_matches_torch_plan(world, E, T, K):
    """ep_sort is torch's stable argsort by expert; ep_routes gives push_plan's destinations,
    sources, offs and row count, and the scatter addresses base[src] + src_pos * row_bytes, for every
    rank of a simulated group (one GPU: no peer memory is touched)."""
    from cutlass_op.bf16_grouped_mm.expert_parallel import push_plan, route_tokens

    dev = torch.device("cuda", 0)
    el = E // world
    idxs = [route_tokens(T, E, K, "zipf", seed=70 + r, device=dev) for r in range(world)]
    sorts = [torch.ops.grouped_mm.ep_sort(i, E, K) for i in idxs]
    for i, (order, inv, tok, es, counts) in zip(idxs, sorts):
        flat = i.reshape(-1)
        ref = torch.argsort(flat, stable=True)
        assert torch.equal(order, ref) and torch.equal(tok, ref // K) and torch.equal(es, flat[ref])
        assert torch.equal(inv[order], torch.arange(flat.numel(), device=dev))
        assert torch.equal(counts, torch.bincount(flat, minlength=E))
    c_all = torch.stack([s_[4] for s_ in sorts])
    cap = T * K * world
    bases = torch.tensor([(1 << 40) + (r << 32) for r in range(world)], dtype=torch.int64, device=dev)
    gbases = bases + (1 << 36)
    for r in range(world):
        es = sorts[r][3]
        ref = push_plan(c_all, es, r, world, el, cap)
        got = torch.ops.grouped_mm.ep_routes(c_all, es, r, cap, bases, gbases, 5760)
        n_recv = int(ref["n_recv"])
        assert torch.equal(got[0], ref["dst_rank"]) and torch.equal(got[1], ref["dst_row"])
        assert torch.equal(got[4], ref["offs"]) and int(got[5]) == n_recv
        assert torch.equal(got[2][:n_recv], ref["src_rank"][:n_recv])
        assert torch.equal(got[3][:n_recv], ref["src_pos"][:n_recv])
        assert (got[2][n_recv:] == -1).all() and (got[6][n_recv:] == 0).all() and (got[7][n_recv:] == 0).all()
        want = bases[ref["src_rank"][:n_recv]] + ref["src_pos"][:n_recv] * 5760
        assert torch.equal(got[6][:n_recv], want) and torch.equal(got[7][:n_recv], want + (1 << 36))


def test_scatter_epilogue_writes_rows_to_their_addresses():
    """mm_scatter (BIAS epilogue with per-row destination addresses) stores exactly what the plain
    operator computes, row by row at the given addresses (a permutation of a local buffer here,
    32- and 16-byte aligned rows), and leaves rows with address 0 alone."""
    from cutlass_op.bf16_grouped_mm.workloads import small_case

    x, w_up, b_up, w_down, b_down, offs, gout = small_case(3, 128, 64, [70, 0, 131], seed=31)
    s = x[:, :64].contiguous().cuda()
    wd, bd, offs = w_down.cuda(), b_down.cuda(), offs.cuda()
    ref = torch.ops.grouped_mm.mm(s, wd, offs, bd, -1)
    M, H_ = s.shape[0], wd.shape[2]
    for pitch in (H_, H_ + 8):  # 256-byte rows (32-byte aligned) and 272-byte rows (16-byte aligned)
        dst = torch.full((M + 5, pitch), float("nan"), dtype=torch.bfloat16, device="cuda")
        perm = torch.randperm(M + 5, generator=torch.Generator().manual_seed(pitch))[:M].cuda()
        ptrs = dst.data_ptr() + perm * (pitch * 2)
        ptrs[7] = 0  # row 7 has no destination
        torch.ops.grouped_mm.mm_scatter(s, wd, offs, bd, ptrs)
        torch.cuda.synchronize()
        got = dst[perm][:, :H_]
        keep = torch.ones(M, dtype=torch.bool)
        keep[7] = False
        assert torch.equal(got[keep.cuda()], ref[keep.cuda()])
        assert torch.isnan(dst[perm[7]].float()).all()
    from cutlass_op.bf16_grouped_mm import check_device_status

    check_device_status()
