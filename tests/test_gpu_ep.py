"""Expert parallelism with the fused CUDA FFN: one GPU in-process, two GPUs (NCCL) when visible."""

from __future__ import annotations

import os
import socket

import pytest
import torch

from oracle import moe_ffn as O

pytestmark = pytest.mark.gpu

E, H, I, T, K = 8, 256, 128, 300, 4


def _reference_ffn(x, idx, wu, bu, wd, bd):
    """Non-EP oracle: every routed copy through its expert (kernel_chain rounding), summed per token."""
    flat = idx.reshape(-1)
    order = torch.argsort(flat, stable=True)
    counts = torch.bincount(flat, minlength=wu.shape[0])
    offs = torch.cumsum(counts, 0).to(torch.int32)
    rows = x[torch.div(order, idx.shape[1], rounding_mode="floor")]
    g = torch.zeros(rows.shape[0], wd.shape[-1], dtype=torch.bfloat16)
    ref = O.kernel_chain(rows, wu, bu, wd, bd, offs, g)
    y = ref["out"]
    out = torch.zeros(x.shape[0], x.shape[1]).index_add(0, torch.div(order, idx.shape[1], rounding_mode="floor"), y)
    return out


def test_ep_world1_matches_oracle():
    from cutlass_op.bf16_grouped_mm.expert_parallel import EPMoEFFN, route_tokens

    dev = torch.device("cuda", 0)
    ffn = EPMoEFFN(E, H, I, device=dev, seed=5)
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    idx = route_tokens(T, E, K, "zipf", seed=2)
    xd = x.to(dev).requires_grad_(True)
    out = ffn(xd, idx.to(dev))
    out.float().sum().backward()
    torch.cuda.synchronize()
    ref = _reference_ffn(x, idx, ffn.w_up.detach().cpu(), ffn.b_up.detach().cpu(), ffn.w_down.detach().cpu(),
                         ffn.b_down.detach().cpu())
    r = O.check("ep_out", out.float().cpu(), ref)
    assert r["ok"], r
    for p in (xd.grad, ffn.w_up.grad, ffn.b_up.grad, ffn.w_down.grad, ffn.b_down.grad):
        assert p is not None and torch.isfinite(p.float()).all()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _ep_worker(rank, world, port, q):
    try:
        _ep_worker_body(rank, world, port, q)
    except Exception:  # report instead of leaving the parent waiting
        import traceback

        q.put((rank, "error", traceback.format_exc()))


def _ep_worker_body(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    from conftest import PKG  # noqa: F401

    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        from cutlass_op.bf16_grouped_mm.expert_parallel import EPMoEFFN, route_tokens

        ffn = EPMoEFFN(E, H, I, device=dev, seed=5, transport="nccl")
        x = torch.randn(T, H, generator=torch.Generator().manual_seed(10 + rank)).to(torch.bfloat16)
        idx = route_tokens(T, E, K, "uniform", seed=20 + rank)
        out = ffn(x.to(dev), idx.to(dev))
        torch.cuda.synchronize()
        # gather every rank's weights so rank 0 can check against a single-process oracle
        ws = [p.detach() for p in (ffn.w_up, ffn.b_up, ffn.w_down, ffn.b_down)]
        gathered = []
        for w in ws:
            parts = [torch.empty_like(w) for _ in range(world)]
            dist.all_gather(parts, w)
            gathered.append(torch.cat(parts, 0).cpu().float().numpy())
        q.put((rank, x.float().numpy(), idx.numpy(), out.detach().float().cpu().numpy(), gathered))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_world2_nccl_matches_oracle():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ep_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(2):
            r = q.get(timeout=240)
            assert not (isinstance(r[1], str) and r[1] == "error"), r[2]
            res[r[0]] = r
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for p in procs:
        assert p.exitcode == 0
    for rank in range(2):
        _, x, idx, out, ws = res[rank]
        wts = [torch.from_numpy(w).to(torch.bfloat16) for w in ws]
        ref = _reference_ffn(torch.from_numpy(x).to(torch.bfloat16), torch.from_numpy(idx), *wts)
        r = O.check(f"ep_out_rank{rank}", torch.from_numpy(out), ref)
        assert r["ok"], r


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
            for transport in ("nccl", "peer", "peer_overlap"):
                ffn = EPMoEFFN(E, H, I, device=dev, seed=5, transport=transport.split("_")[0],
                               overlap=transport.endswith("overlap"))
                x = torch.randn(T, H, generator=torch.Generator().manual_seed(10 + rank)).to(torch.bfloat16)
                x = x.to(dev).requires_grad_(True)
                idx = route_tokens(T, E, K, "zipf", seed=20 + rank).to(dev)
                w = torch.rand(T, K, generator=torch.Generator().manual_seed(30 + rank)).to(dev)
                for step in range(2):  # second step reuses the peer buffers
                    x.grad = None
                    ffn.zero_grad()
                    out = ffn(x, idx, w)
                    g = torch.randn(T, H, generator=torch.Generator().manual_seed(40 + rank + step)).to(torch.bfloat16)
                    out.backward(g.to(dev))
                torch.cuda.synchronize()
                res[transport] = [t.detach().float().cpu().numpy() for t in
                                  (out, x.grad, ffn.w_up.grad, ffn.b_up.grad, ffn.w_down.grad, ffn.b_down.grad)]
            q.put((rank, res))
        finally:
            dist.destroy_process_group()
    except Exception:
        import traceback

        q.put((rank, "error", traceback.format_exc()))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_world2_peer_transport_matches_nccl():
    """Dispatch/combine as peer-memory pushes gives the NCCL all-to-all path's outputs and gradients;
    with the dispatch-gradient push overlapped, bit-identical ones."""
    import torch.multiprocessing as mp

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
    names = ["out", "dx", "dw_up", "db_up", "dw_down", "db_down"]
    for rank in range(2):
        for name, a, b in zip(names, res[rank]["peer"], res[rank]["nccl"]):
            r = O.check(f"rank{rank}:{name}", torch.from_numpy(a), torch.from_numpy(b))
            assert r["ok"], r
        # the overlapped dispatch-gradient push changes the timing, not one bit of the results
        for name, a, b in zip(names, res[rank]["peer_overlap"], res[rank]["peer"]):
            assert (a == b).all(), f"rank{rank}:{name}: overlap changed the result"
