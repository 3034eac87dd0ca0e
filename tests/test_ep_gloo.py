"""Expert-parallel dispatch/combine on CPU ranks (gloo, world size 2).

The expert compute is the fp32 oracle composition (the fused CUDA FFN needs a GPU); the test covers
the routing, count exchange, uneven all-to-alls, the (rank, expert) -> expert-order permutation that
builds `offs`, the combine, and the gradients through all of it, against one process computing the
same MoE over every rank's tokens with all experts.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

E, H, I, T, K = 8, 32, 16, 24, 2
WORLD = 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _inputs(rank):
    g = torch.Generator().manual_seed(100 + rank)
    x = torch.randn(T, H, generator=g)
    from cutlass_op.bf16_grouped_mm.expert_parallel import route_tokens

    idx = route_tokens(T, E, K, "zipf" if rank == 0 else "uniform", seed=rank)
    w = torch.rand(T, K, generator=g)
    return x, idx, w


def _weights():
    g = torch.Generator().manual_seed(7)
    wu = torch.randn(E, H, 2 * I, generator=g) / H ** 0.5
    bu = torch.randn(E, 2 * I, generator=g) * 0.02
    wd = torch.randn(E, I, H, generator=g) / I ** 0.5
    bd = torch.randn(E, H, generator=g) * 0.02
    return wu, bu, wd, bd


def _ffn(r, e, wu, bu, wd, bd):
    from oracle.moe_ffn import swiglu_fwd

    return swiglu_fwd(r @ wu[e] + bu[e]) @ wd[e] + bd[e]


def _worker(rank, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import sys

    from conftest import PKG, REPO  # noqa: F401  (puts the package on sys.path)

    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        from cutlass_op.bf16_grouped_mm.expert_parallel import ep_moe_ffn

        wu, bu, wd, bd = _weights()
        el = E // WORLD
        sl = slice(rank * el, (rank + 1) * el)
        local = [t[sl].clone().requires_grad_(True) for t in (wu, bu, wd, bd)]
        x, idx, w = _inputs(rank)
        x = x.clone().requires_grad_(True)

        def expert_fn(rows, offs):
            outs, prev = [], 0
            for e, end in enumerate(offs.tolist()):
                outs.append(_ffn(rows[prev:end], e, *local))
                prev = end
            return torch.cat(outs, 0) if outs else rows.new_zeros(0, H)

        out, plan = ep_moe_ffn(x, idx, E, expert_fn, router_weights=w)
        gout = torch.randn(T, H, generator=torch.Generator().manual_seed(300 + rank))
        out.backward(gout)
        # numpy arrays travel by value (torch tensors would share memory with an exiting process)
        q.put((rank, out.detach().numpy(), x.grad.numpy(), [t.grad.numpy() for t in local], plan.offs.tolist(),
               plan.send_splits, plan.recv_splits))
    finally:
        dist.destroy_process_group()


def _reference():
    wu, bu, wd, bd = [t.clone().requires_grad_(True) for t in _weights()]
    outs, xs = [], []
    for rank in range(WORLD):
        x, idx, w = _inputs(rank)
        x = x.clone().requires_grad_(True)
        out = torch.zeros(T, H)
        for t in range(T):
            for j in range(K):
                out[t] = out[t] + w[t, j] * _ffn(x[t:t + 1], int(idx[t, j]), wu, bu, wd, bd)[0]
        out.backward(torch.randn(T, H, generator=torch.Generator().manual_seed(300 + rank)))
        outs.append(out.detach())
        xs.append(x.grad)
    return outs, xs, [wu.grad, bu.grad, wd.grad, bd.grad]


def test_ep_dispatch_combine_world2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(WORLD):
        r = q.get(timeout=120)
        results[r[0]] = r
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    ref_out, ref_dx, ref_dw = _reference()
    el = E // WORLD
    total_recv = 0
    for rank in range(WORLD):
        _, out, dx, dws, offs, send, recv = results[rank]
        out, dx, dws = torch.from_numpy(out), torch.from_numpy(dx), [torch.from_numpy(v) for v in dws]
        assert torch.allclose(out, ref_out[rank], atol=1e-4, rtol=1e-4)
        assert torch.allclose(dx, ref_dx[rank], atol=1e-4, rtol=1e-4)
        for got, ref in zip(dws, ref_dw):
            assert torch.allclose(got, ref[rank * el:(rank + 1) * el], atol=1e-4, rtol=1e-4)
        assert sum(send) == T * K
        assert offs[-1] == sum(recv)
        total_recv += sum(recv)
    assert total_recv == WORLD * T * K


def test_dispatch_plan_single_rank():
    """World size 1: the plan is a pure local sort; offs are the per-expert counts' cumsum."""
    from cutlass_op.bf16_grouped_mm.expert_parallel import DispatchPlan, route_tokens

    idx = route_tokens(50, 6, 3, "zipf", seed=3)
    plan = DispatchPlan(idx, 6, 1)
    counts = torch.bincount(idx.reshape(-1), minlength=6)
    assert plan.offs.tolist() == torch.cumsum(counts, 0).tolist()
    assert plan.send_splits == [150] and plan.recv_splits == [150]
    # rows in expert order: the expert id of every copy is non-decreasing
    flat = idx.reshape(-1)[plan.order]
    assert torch.all(flat[1:] >= flat[:-1])


def test_route_tokens_distinct_experts():
    from cutlass_op.bf16_grouped_mm.expert_parallel import route_tokens

    idx = route_tokens(1000, 16, 4, "zipf", seed=1)
    assert idx.shape == (1000, 4)
    assert all(len(set(r)) == 4 for r in idx.tolist())


def test_world1_identity_experts_sum_copies():
    """Without a process group the exchange is local; identity experts return k copies summed."""
    from cutlass_op.bf16_grouped_mm.expert_parallel import ep_moe_ffn

    if dist.is_initialized():
        pytest.skip("process group already initialised")
    x = torch.randn(5, 3)
    idx = torch.tensor([[0, 2], [1, 2], [2, 0], [1, 0], [0, 1]])
    out, plan = ep_moe_ffn(x, idx, 3, lambda r, o: r)
    assert torch.allclose(out, 2 * x)
    assert plan.offs.tolist() == [4, 7, 10]


@pytest.mark.parametrize("world,E,T,K", [(2, 8, 24, 2), (4, 8, 50, 3), (3, 6, 7, 2)])
def test_push_plan_is_a_consistent_exchange(world, E, T, K):
    """Simulate every rank of the peer transport in one process: the destination map (source side) and
    the source map (owner side) are inverse to each other, rows land expert-major then source-major,
    and the owner's offs count exactly the rows it receives."""
    from cutlass_op.bf16_grouped_mm.expert_parallel import push_plan, route_tokens

    el = E // world
    idx = [route_tokens(T, E, K, "zipf" if r % 2 else "uniform", seed=10 + r) for r in range(world)]
    flats = [i.reshape(-1) for i in idx]
    orders = [torch.argsort(f, stable=True) for f in flats]
    c_all = torch.stack([torch.bincount(f, minlength=E) for f in flats])
    cap = T * K * world
    plans = [push_plan(c_all, flats[r][orders[r]], r, world, el, cap) for r in range(world)]
    # push: owner o's row (dst_row) receives (source s, sorted copy p)
    received = [dict() for _ in range(world)]
    for s in range(world):
        for p in range(T * K):
            o, row = int(plans[s]["dst_rank"][p]), int(plans[s]["dst_row"][p])
            assert 0 <= row < cap and (row not in received[o])
            received[o][row] = (s, p)
    for o in range(world):
        n = int(plans[o]["n_recv"][0])
        assert sorted(received[o]) == list(range(n))
        assert plans[o]["offs"].tolist() == torch.cumsum(c_all[:, o * el:(o + 1) * el].sum(0), 0).tolist()
        for row in range(n):
            s, p = received[o][row]
            assert int(plans[o]["src_rank"][row]) == s and int(plans[o]["src_pos"][row]) == p
        # expert-major, then source-major order
        keys = []
        for row in range(n):
            s, p = received[o][row]
            e = int(flats[s][orders[s][p]])
            assert e // el == o
            keys.append((e, s, p))
        assert keys == sorted(keys)


def test_ep_oracle_matches_direct_autograd():
    """oracle.ep_ffn.ep_reference (the checker of the GPU expert-parallel tests) against a direct
    fp32 per-token autograd computation over two ranks' tokens."""
    from oracle import moe_ffn as O
    from oracle.ep_ffn import ep_reference
    from cutlass_op.bf16_grouped_mm.expert_parallel import route_tokens

    bf = torch.bfloat16
    wts = [t.to(bf) for t in _weights()]
    xs, idxs, ws, gs = [], [], [], []
    for r in range(2):
        g = torch.Generator().manual_seed(300 + r)
        xs.append(torch.randn(T, H, generator=g).to(bf))
        idxs.append(route_tokens(T, E, K, "zipf", seed=40 + r))
        ws.append(torch.rand(T, K, generator=g))
        gs.append(torch.randn(T, H, generator=g).to(bf))
    want = ep_reference(xs, idxs, ws, gs, *wts)
    leaves = [t.float().requires_grad_(True) for t in wts]
    for r in range(2):
        x = xs[r].float().requires_grad_(True)
        w = ws[r].clone().requires_grad_(True)
        out = torch.stack([sum(w[t, j] * _ffn(x[t:t + 1], int(idxs[r][t, j]), *leaves)[0] for j in range(K))
                           for t in range(T)])
        (out * gs[r].float()).sum().backward()
        for name, a, b in (("out", want["out"][r], out.detach()), ("dx", want["dx"][r], x.grad),
                           ("dw_router", want["dw_router"][r], w.grad)):
            res = O.check(f"rank{r}:{name}", a, b)
            assert res["ok"], res
    for name, p in zip(("dw_up", "db_up", "dw_down", "db_down"), leaves):
        res = O.check(name, want[name], p.grad)
        assert res["ok"], res
