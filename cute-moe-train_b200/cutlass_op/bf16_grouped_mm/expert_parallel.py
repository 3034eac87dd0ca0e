"""Expert parallelism for the fused MoE FFN: E/N experts per GPU, tokens exchanged with all-to-all.

The reference has no distributed code (its numbers were taken under FSDP without expert
parallelism, README.md:81-84; compute/communication overlap is on its roadmap, README.md:103-107).
This module shards the experts over the ranks of a process group, one process per GPU:

forward
  1. every routed copy (token t, slot j) of the local tokens goes to expert e = expert_idx[t, j],
     owned by rank e // (E/N); copies are sorted by expert, which also groups them by rank;
  2. per-(rank, expert) counts are exchanged with a small all-to-all;
  3. token rows are exchanged with ``all_to_all_single`` (uneven splits) -- dispatch;
  4. received rows are permuted from (source rank, expert) order into expert order, which yields
     the int32 ``offs`` of the grouped GEMMs;
  5. the fused FFN runs on the local experts (grouped_mm_swiglu -> grouped_mm_downproj);
  6. results return with the inverse all-to-all (combine) and are summed over the top-k slots,
     optionally weighted by the router probabilities.
backward mirrors it: the all-to-alls are differentiable (their gradient is the reverse exchange) and
the expert weight gradients stay local -- pure EP needs no gradient all-reduce.

Two transports carry the rows.  ``ep_moe_ffn`` (above; CPU/gloo and ``transport="nccl"``) uses NCCL
all-to-alls with host-side split sizes.  ``ep_moe_ffn_peer`` (CUDA, the default of ``EPMoEFFN``) has
each source rank write its rows straight into the owners' receive buffers through CUDA IPC mappings
(``grouped_mm::push_rows``: plain peer stores, no TMA, no multicast), with the whole plan computed on
the device; each push signals its completion through per-rank flags in peer memory and the readers
wait on their own flags (no collective barrier).  No kernel reads a peer's memory.
``expert_fn`` can replace the fused FFN (e.g. with a CPU reference for gloo tests of the routing).
"""

from __future__ import annotations

import math
from typing import Callable

import torch
import torch.distributed as dist

from .optimer import timed


def route_tokens(tokens: int, num_experts: int, topk: int, routing: str = "zipf", seed: int = 0,
                 device="cpu", zipf_s: float = 1.1) -> torch.Tensor:
    """Seeded synthetic router: [tokens, topk] distinct expert ids per token.

    ``uniform`` draws k distinct experts uniformly; ``zipf`` weights expert popularity with
    Zipf(zipf_s) over a seeded permutation (Gumbel top-k = sampling without replacement).
    """
    g = torch.Generator(device="cpu").manual_seed(seed)
    if routing == "uniform":
        logw = torch.zeros(num_experts)
    else:
        perm = torch.randperm(num_experts, generator=g)
        w = torch.arange(1, num_experts + 1, dtype=torch.float64).pow(-zipf_s)
        weights = torch.zeros(num_experts, dtype=torch.float64)
        weights[perm] = w
        logw = torch.log(weights).float()
    u = torch.rand(tokens, num_experts, generator=g).clamp_(1e-12, 1.0 - 1e-7)
    keys = logw.unsqueeze(0) - torch.log(-torch.log(u))
    return keys.topk(topk, dim=1).indices.to(device)


class DispatchPlan:
    """Host-side bookkeeping of one dispatch: split sizes and the permutations on the device."""

    def __init__(self, expert_idx: torch.Tensor, num_experts: int, world: int, group=None):
        device = expert_idx.device
        T, k = expert_idx.shape
        self.tokens, self.topk = T, k
        e_local = num_experts // world
        self.e_local = e_local
        flat = expert_idx.reshape(-1).to(torch.int64)
        # stable sort of the T*k copies by expert id (=> grouped by destination rank as well)
        self.order = torch.argsort(flat, stable=True)
        self.copy_token = torch.div(self.order, k, rounding_mode="floor")
        self.inv_order = _inverse(self.order)                             # copy (t*k + j) -> sorted position
        counts_e = torch.bincount(flat, minlength=num_experts)            # [E] copies per expert
        send_counts = counts_e.view(world, e_local)                       # [dest rank, local expert]
        recv_counts = torch.empty_like(send_counts)
        if world > 1:
            dist.all_to_all_single(recv_counts.view(-1), send_counts.reshape(-1).contiguous(), group=group)
        else:
            recv_counts.copy_(send_counts)
        # One device->host read of the split sizes (all_to_all_single takes host lists).
        both = torch.stack([send_counts.sum(1), recv_counts.sum(1)]).cpu()
        self.send_splits = [int(v) for v in both[0]]
        self.recv_splits = [int(v) for v in both[1]]
        self.recv_counts = recv_counts                                    # [src rank, local expert]
        n_recv = sum(self.recv_splits)
        self.n_recv = n_recv
        # received rows are ordered (src rank, expert); the GEMMs want (expert, src rank)
        seg_key = (torch.arange(e_local, device=device).unsqueeze(0) * world
                   + torch.arange(world, device=device).unsqueeze(1))     # [src, expert] -> e*world + src
        row_key = torch.repeat_interleave(seg_key.reshape(-1), recv_counts.reshape(-1), output_size=n_recv)
        self.to_expert_order = torch.argsort(row_key, stable=True)        # expert-ordered row -> received row
        self.from_expert_order = _inverse(self.to_expert_order)
        self.identity_order = world == 1                                  # received order is expert order
        per_expert = recv_counts.sum(0)                                   # [local expert]
        self.offs = torch.cumsum(per_expert, 0).to(torch.int32)
        self.local_rows = n_recv


def _inverse(perm: torch.Tensor) -> torch.Tensor:
    inv = torch.empty_like(perm)
    inv[perm] = torch.arange(perm.numel(), device=perm.device, dtype=perm.dtype)
    return inv


# Row movement.  CUDA tensors go through the grouped_mm::gather_rows / combine_rows kernels (one
# HBM pass each, fp32 accumulation in the combine); the torch expressions below serve CPU tensors,
# i.e. the process-group tests of the routing logic that run on CPU ranks.
def _gather(src, idx, scale=None):
    if src.is_cuda:
        return torch.ops.grouped_mm.gather_rows(src, idx, scale)
    out = src[idx]
    return out if scale is None else (out.float() * scale.float().unsqueeze(1)).to(src.dtype)


def _combine(rows, pos, weights, k):
    if rows.is_cuda:
        return torch.ops.grouped_mm.combine_rows(rows, pos, weights, k)
    g = rows[pos].float().view(-1, k, rows.shape[1])
    if weights is not None:
        g = g * weights.float().view(-1, k, 1)
    return g.sum(1).to(rows.dtype)


class _Dispatch(torch.autograd.Function):
    """Token copies in sorted-by-expert order: out[p] = x[copy_token[p]]."""

    @staticmethod
    def forward(ctx, x, copy_token, inv_order, k):
        ctx.save_for_backward(inv_order)
        ctx.k = k
        with timed("ep_dispatch_gather"):
            return _gather(x, copy_token)

    @staticmethod
    def backward(ctx, g):
        (inv_order,) = ctx.saved_tensors
        with timed("ep_dispatch_gather_bwd"):
            return _combine(g.contiguous(), inv_order, None, ctx.k), None, None, None


class _Permute(torch.autograd.Function):
    """out[i] = x[perm[i]] for a permutation; the gradient moves back with the inverse."""

    @staticmethod
    def forward(ctx, x, perm, inv_perm):
        ctx.save_for_backward(inv_perm)
        with timed("ep_permute"):
            return _gather(x, perm)

    @staticmethod
    def backward(ctx, g):
        (inv_perm,) = ctx.saved_tensors
        with timed("ep_permute_bwd"):
            return _gather(g.contiguous(), inv_perm), None, None


class _Combine(torch.autograd.Function):
    """out[t] = sum_j w[t, j] * ret[inv_order[t*k + j]] (w = 1 when absent), fp32 accumulation."""

    @staticmethod
    def forward(ctx, ret, inv_order, copy_token, order, w_flat, k):
        ctx.save_for_backward(ret, inv_order, copy_token, order, w_flat if w_flat is not None else ret.new_empty(0))
        ctx.k, ctx.has_w = k, w_flat is not None
        with timed("ep_combine"):
            return _combine(ret, inv_order, w_flat, k)

    @staticmethod
    def backward(ctx, g):
        ret, inv_order, copy_token, order, w_flat = ctx.saved_tensors
        g = g.contiguous()
        scale = w_flat[order] if ctx.has_w else None
        with timed("ep_combine_bwd"):
            grad_ret = _gather(g, copy_token, scale)
        grad_w = None
        if ctx.has_w and ctx.needs_input_grad[4]:
            copies = ret[inv_order].float().view(-1, ctx.k, ret.shape[1])
            grad_w = (copies * g.float().unsqueeze(1)).sum(-1).reshape(-1)
        return grad_ret, None, None, None, grad_w, None


def _exchange(x: torch.Tensor, out_splits, in_splits, group, name) -> torch.Tensor:
    out = x.new_empty((sum(out_splits),) + tuple(x.shape[1:]))
    with timed(name):
        dist.all_to_all_single(out, x.contiguous(), out_splits, in_splits, group=group)
    return out


class _AllToAll(torch.autograd.Function):
    """Uneven all-to-all of rows; its gradient is the same exchange with the splits swapped."""

    @staticmethod
    def forward(ctx, x, out_splits, in_splits, group):
        ctx.out_splits, ctx.in_splits, ctx.group = out_splits, in_splits, group
        return _exchange(x, out_splits, in_splits, group, "ep_all_to_all")

    @staticmethod
    def backward(ctx, g):
        return _exchange(g, ctx.in_splits, ctx.out_splits, ctx.group, "ep_all_to_all_bwd"), None, None, None


def _all_to_all(x: torch.Tensor, out_splits, in_splits, group) -> torch.Tensor:
    return _AllToAll.apply(x, out_splits, in_splits, group)


def ep_moe_ffn(x: torch.Tensor, expert_idx: torch.Tensor, num_experts: int, expert_fn: Callable,
               group=None, router_weights: torch.Tensor | None = None,
               plan: DispatchPlan | None = None) -> tuple[torch.Tensor, DispatchPlan]:
    """Expert-parallel MoE FFN over the ranks of ``group``.

    x: [T, H] local tokens; expert_idx: [T, k] global expert ids; expert_fn(rows, offs) -> [rows, H]
    runs the local experts on expert-ordered rows.  Returns ([T, H] combined output, plan).
    """
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if num_experts % world:
        raise RuntimeError(f"num_experts ({num_experts}) must be divisible by the world size ({world})")
    if plan is None:
        with timed("ep_plan"):
            plan = DispatchPlan(expert_idx, num_experts, world, group)
    k = plan.topk
    send = _Dispatch.apply(x, plan.copy_token, plan.inv_order, k)        # [T*k, H] sorted by expert
    recv = _all_to_all(send, plan.recv_splits, plan.send_splits, group) if world > 1 else send
    rows = recv if plan.identity_order else _Permute.apply(recv, plan.to_expert_order, plan.from_expert_order)
    y = expert_fn(rows, plan.offs)
    back = y if plan.identity_order else _Permute.apply(y, plan.from_expert_order, plan.to_expert_order)
    ret = _all_to_all(back, plan.send_splits, plan.recv_splits, group) if world > 1 else back
    w_flat = router_weights.reshape(-1).float() if router_weights is not None else None
    out = _Combine.apply(ret, plan.inv_order, plan.copy_token, plan.order, w_flat, k)
    return out, plan


# ============================================================================ peer-memory transport
#
# The NCCL path above moves every row three times per direction (gather into a send buffer, the
# all-to-all, a permutation into expert order).  The peer path writes each row once, straight into
# its final place in another GPU's memory: every rank owns four receive buffers, shared with all
# ranks of the group through CUDA IPC once (no multicast object):
#   rows  [cap, H]   expert-ordered token rows of this rank's experts   (forward dispatch target)
#   ret   [T*k, H]   expert outputs of this rank's token copies, sorted (forward combine target)
#   grows [cap, H]   gradients of `rows`                                 (backward of the combine)
#   gret  [T*k, H]   gradients of this rank's token copies               (backward of the dispatch)
# cap = ceil(capacity_factor * T*k) rows, the most one rank can receive (rows past it are skipped
# and reported through the device status word, MGF_DEV_ROW_OUT_OF_RANGE).  All destination rows
# are computed on the device from the all-gathered (source rank, expert) count matrix, so no split
# size is read on the host.  Each push signals its completion through the ranks' flag arrays and
# the readers wait on their own flags; the count all-gather at the start of a call orders it after
# every rank's use of the buffers in the previous call.


def push_plan(c_all: torch.Tensor, e_sorted: torch.Tensor, rank: int, world: int, e_local: int, cap: int) -> dict:
    """Destination and source maps of the peer transport, on the device (no host synchronisation).

    c_all: [world, E] copies from source rank s to expert e; e_sorted: this rank's copy experts in
    sorted order.  Returns
      dst_rank/dst_row [T*k]: where sorted copy p of this rank lands (owner rank, row of its `rows`);
      src_rank/src_pos [cap]: for row j of this rank's `rows`, the source rank and its sorted copy;
      offs [e_local] int32 and n_recv [1] int32 of the received rows.
    Owner row layout: local expert-major, source rank next, the source's copies in sorted order.
    """
    dev = c_all.device
    E = c_all.shape[1]
    n = e_sorted.numel()
    ex = lambda t, d: t.cumsum(d) - t  # noqa: E731  exclusive cumulative sum
    pos = ex(c_all, 1)                                           # [world, E] first sorted copy per expert
    tot = c_all.sum(0)                                           # [E] rows of each expert
    base = ex(tot.view(world, e_local), 1).reshape(E)            # expert's first row within its owner
    before = ex(c_all, 0)                                        # [world, E] rows from lower source ranks
    within = torch.arange(n, device=dev) - pos[rank][e_sorted]
    dst_row = base[e_sorted] + before[rank][e_sorted] + within
    dst_rank = torch.div(e_sorted, e_local, rounding_mode="floor")
    cl = c_all[:, rank * e_local:(rank + 1) * e_local]          # [world, e_local]
    seg = cl.t().reshape(-1)                                     # (local expert, source) segments
    seg_end = seg.cumsum(0)
    seg_start = seg_end - seg
    j = torch.arange(cap, device=dev)
    sid = torch.searchsorted(seg_end, j, right=True).clamp_(max=seg.numel() - 1)
    e_l = torch.div(sid, world, rounding_mode="floor")
    src = sid - e_l * world
    src_pos = pos[src, rank * e_local + e_l] + (j - seg_start[sid])
    offs = cl.sum(0).cumsum(0).to(torch.int32)
    return {"dst_rank": dst_rank.contiguous(), "dst_row": dst_row.contiguous(), "src_rank": src.contiguous(),
            "src_pos": src_pos.contiguous(), "offs": offs, "n_recv": offs[-1:].contiguous()}


class PeerBuffers:
    """Receive buffers shared with every rank of `group` through CUDA IPC (allocated once), plus the
    completion flags of the pushes.

    Each rank owns a uint64 flag array [world], IPC-shared like the buffers: a push launch with
    sequence number q writes q into slot `rank` of every rank's flags once all of its rows are
    visible (mgf_push_rows' completion signal), and a reader waits on its own array until every slot
    holds q (mgf_wait_flags).  Every rank issues the same pushes in the same order, so the sequence
    numbers agree without any exchange."""

    WAIT_TIMEOUT_NS = int(float(__import__("os").environ.get("MGF_EP_WAIT_TIMEOUT_S", "5")) * 1e9)

    def __init__(self, shapes: dict, dtype, device, group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.local = {k: torch.empty(v, dtype=dtype, device=device) for k, v in shapes.items()}
        self.flags = torch.zeros(self.world, dtype=torch.int64, device=device)
        self.next_rank = torch.full((1,), (self.rank + 1) % self.world, dtype=torch.int64, device=device)
        self.counters = torch.zeros(4, dtype=torch.int64, device=device)  # one per push kind
        self.seq = 0
        from ._ext import ipc_handle

        shared = dict(self.local, flags=self.flags)
        handles = {k: ipc_handle(t.data_ptr()) for k, t in shared.items()}
        everyone = [None] * self.world
        dist.all_gather_object(everyone, handles, group=group)
        # Open every peer allocation with THIS rank's device current (mgf_ipc_open), so this device
        # gets peer access to it; torch's own IPC path would map it into the peer device's context.
        # Buffers carved from one allocation segment share a handle: open each handle once.
        from ._ext import ipc_open

        self._opened = {}
        self.bases = {}
        for k, t in shared.items():
            ptrs = []
            for r in range(self.world):
                if r == self.rank:
                    ptrs.append(t.data_ptr())
                    continue
                handle, offset = everyone[r][k]
                if handle not in self._opened:
                    self._opened[handle] = ipc_open(handle)
                ptrs.append(self._opened[handle] + offset)
            self.bases[k] = torch.tensor(ptrs, dtype=torch.int64, device=device)
        self.side_stream = torch.cuda.Stream(device=device)
        torch.cuda.synchronize(device)
        dist.barrier(group=group)  # every rank's flags are mapped (and zero) before the first signal

    def close(self):
        from ._ext import ipc_close

        torch.cuda.synchronize()
        for base in self._opened.values():
            ipc_close(base)
        self._opened = {}

    def push(self, kind: int, src, src_idx, scale, n_dev, dst_rank, dst_row, target: str, dst_rows: int, n_max: int):
        """One push into every rank's `target` buffer followed, on the same stream, by the wait for all
        ranks' pushes of this round: afterwards this rank's own `target`-side data is complete."""
        self.wait(self.push_async(kind, src, src_idx, scale, n_dev, dst_rank, dst_row, target, dst_rows, n_max))

    def push_async(self, kind: int, src, src_idx, scale, n_dev, dst_rank, dst_row, target: str, dst_rows: int,
                   n_max: int, rotate: torch.Tensor | None = None) -> int:
        """The push of push() without the wait, on the current stream; returns its sequence number.
        Entries sorted by destination rank are visited from the first one bound for the next rank
        (`rotate`, default: counted from dst_rank on the device), so the ranks' pushes start on
        different destinations instead of all on rank 0."""
        self.seq += 1
        if rotate is None and n_dev is None:
            rotate = (dst_rank < self.next_rank).sum().view(1)
        torch.ops.grouped_mm.push_rows(src, src_idx, scale, n_dev, dst_rank, dst_row, self.bases[target], dst_rows,
                                       src.shape[1], n_max, self.bases["flags"], self.counters[kind:kind + 1],
                                       self.seq, self.rank, rotate)
        return self.seq

    def signal(self) -> int:
        """Signal, after the stream's earlier work (a scatter-epilogue GEMM that wrote rows into the
        ranks' buffers), the next sequence number to every rank; returns it for wait()."""
        self.seq += 1
        torch.ops.grouped_mm.signal_flags(self.bases["flags"], self.rank, self.seq)
        return self.seq

    def wait(self, seq: int) -> None:
        with timed("ep_peer_wait"):
            torch.ops.grouped_mm.wait_flags(self.flags, seq, self.WAIT_TIMEOUT_NS)


class _PeerState:
    pass


class _PeerDispatch(torch.autograd.Function):
    """x [T, H] -> this rank's expert-ordered rows [cap, H], rows written by their source ranks."""

    @staticmethod
    def forward(ctx, x, st):
        ctx.st = st
        with timed("ep_peer_dispatch"):
            st.bufs.push(0, x.contiguous(), st.copy_token, None, None, st.plan["dst_rank"], st.plan["dst_row"],
                         "rows", st.cap, st.n)
        return st.bufs.local["rows"].view(st.cap, x.shape[1])

    @staticmethod
    def backward(ctx, g_rows):
        st = ctx.st
        if getattr(st, "dispatch_bwd_done", None) is not None:
            # already pushed (and every rank's push awaited) on the side stream by the FFN's backward
            torch.cuda.current_stream().wait_event(st.dispatch_bwd_done)
            st.dispatch_bwd_done = None
        else:
            _push_rows_grad(g_rows, st)
        with timed("ep_combine"):
            gx = torch.ops.grouped_mm.combine_rows(st.bufs.local["gret"], st.inv_order, None, st.k)
        return gx, None


def _push_rows_grad(g_rows: torch.Tensor, st) -> None:
    """Gradient of the dispatch: each received row's gradient goes back to its source's `gret`."""
    with timed("ep_peer_dispatch_bwd"):
        st.bufs.push(3, g_rows.contiguous(), None, None, st.plan["n_recv"], st.plan["src_rank"], st.plan["src_pos"],
                     "gret", st.n, st.cap)


def _start_dispatch_bwd(g_rows: torch.Tensor, st) -> None:
    """Push the rows' gradient and wait for every rank's push on the side stream, so both run under
    the up-projection weight gradient that the expert FFN's backward launches next; the dispatch's
    backward then only waits for the recorded event."""
    side = st.side_stream
    side.wait_stream(torch.cuda.current_stream())
    g_rows.record_stream(side)
    with torch.cuda.stream(side):
        _push_rows_grad(g_rows, st)
        ev = torch.cuda.Event()
        ev.record(side)
    st.dispatch_bwd_done = ev


class _EPExpertFFN(torch.autograd.Function):
    """The local experts' fused FFN (grouped_mm_swiglu -> grouped_mm_downproj) for the peer transport.

    Same launches and results as the two wrappers; the backward hands the received rows' gradient
    to the dispatch push on a side stream as soon as the up-projection dgrad has produced it, before
    launching the up-projection weight gradient, so the NVLink push and its wait overlap that GEMM
    (the push kernel's blocks co-reside with the GEMM's one CTA per SM).
    """

    @staticmethod
    def forward(ctx, rows, w_up, b_up, w_down, b_down, offs, alpha, limit, st):
        with timed("up_swiglu_fwd"):
            s, aux = torch.ops.grouped_mm.mm_swiglu(rows, w_up, offs, b_up, alpha, limit)
        with timed("down_fwd"):
            y = torch.ops.grouped_mm.mm(s, w_down, offs, b_down, -1)
        ctx.save_for_backward(rows, w_up, w_down, s, aux, offs)
        ctx.alpha, ctx.limit, ctx.st = alpha, limit, st
        return y

    @staticmethod
    def backward(ctx, g):
        rows, w_up, w_down, s, aux, offs = ctx.saved_tensors
        g = g.contiguous()
        with timed("down_wgrad_bias"):
            g_wd, g_bd = torch.ops.grouped_mm.mm_wgrad_bias(s.transpose(-2, -1), g, offs)
        with timed("down_dgrad_swiglu_bwd"):
            grad_aux = torch.ops.grouped_mm.mm_swiglu_bwd(g, w_down.transpose(-2, -1), offs, aux, ctx.alpha, ctx.limit)
        with timed("up_dgrad"):
            g_rows = torch.ops.grouped_mm.mm(grad_aux, w_up.transpose(-2, -1), offs, None, -1)
        if ctx.needs_input_grad[0] and ctx.st.overlap:
            _start_dispatch_bwd(g_rows, ctx.st)
        with timed("up_wgrad_bias"):
            g_wu, g_bu = torch.ops.grouped_mm.mm_wgrad_bias(rows.transpose(-2, -1), grad_aux, offs)
        return g_rows, g_wu, g_bu.to(w_up.dtype), g_wd, g_bd.to(w_down.dtype), None, None, None, None


class _PeerCombine(torch.autograd.Function):
    """Expert outputs [cap, H] -> per-token sums [T, H]; rows written back into their sources."""

    @staticmethod
    def forward(ctx, y, w_flat, st):
        ctx.st, ctx.has_w = st, w_flat is not None
        ctx.save_for_backward(w_flat if w_flat is not None else y.new_empty(0))
        with timed("ep_peer_combine"):
            st.bufs.push(1, y.contiguous(), None, None, st.plan["n_recv"], st.plan["src_rank"], st.plan["src_pos"],
                         "ret", st.n, st.cap)
        with timed("ep_combine"):
            return torch.ops.grouped_mm.combine_rows(st.bufs.local["ret"], st.inv_order, w_flat, st.k)

    @staticmethod
    def backward(ctx, g):
        st = ctx.st
        (w_flat,) = ctx.saved_tensors
        g = g.contiguous()
        scale = w_flat[st.order].contiguous() if ctx.has_w else None
        with timed("ep_peer_combine_bwd"):
            st.bufs.push(2, g, st.copy_token, scale, None, st.plan["dst_rank"], st.plan["dst_row"], "grows", st.cap,
                         st.n)
        grad_w = None
        if ctx.has_w and ctx.needs_input_grad[1]:
            copies = st.bufs.local["ret"][st.inv_order].float().view(-1, st.k, g.shape[1])
            grad_w = (copies * g.float().unsqueeze(1)).sum(-1).reshape(-1)
        return st.bufs.local["grows"].view(st.cap, g.shape[1]), grad_w, None


def _split_halves(st) -> dict:
    """The routed copies split by their owner's local-expert half (first e_local/2 experts, then the
    rest), as index arrays for the two-part pushes: first-half entries ascending in destination rank,
    second half flipped (descending); counts and start rotations as device scalars (no host sync)."""
    if getattr(st, "halves", None) is not None:
        return st.halves
    plan = st.plan
    el = plan["offs"].numel()
    h = el // 2
    first = torch.remainder(st.e_sorted, el) < h
    perm = torch.argsort((~first).to(torch.int8), stable=True)  # first-half copies, then the rest
    n_a = first.sum(dtype=torch.int32).view(1)
    nxt = st.bufs.next_rank
    st.halves = {
        "h": h, "perm": perm, "n_a": n_a, "n_b": (st.n - n_a).to(torch.int32),
        "src": st.copy_token[perm], "d_rank": plan["dst_rank"][perm], "d_row": plan["dst_row"][perm],
        "rot_a": (first & (plan["dst_rank"] < nxt)).sum().view(1),
        "rot_b": (~first & (plan["dst_rank"] > nxt)).sum().view(1)}
    return st.halves


def _pipelined_dispatch_up(x, w_up, b_up, st):
    """Dispatch + up-projection in two halves of the local experts, so the second half's rows cross
    NVLink while the first half's GEMM runs: push the copies bound for every owner's first e_local/2
    experts (main stream), push the rest on the side stream, wait for the first push, run the
    up-proj + bias + SwiGLU over experts [0, h), wait for the second push, run it over [h, e_local)
    (mgf_gemm_desc.group_begin) into the same outputs."""
    bufs, plan = st.bufs, st.plan
    offs = plan["offs"]
    el = offs.numel()
    h = el // 2
    n = st.n
    with timed("ep_peer_dispatch"):
        sp = _split_halves(st)
        src, d_rank, d_row, n_a, n_b, rot_a, rot_b = (sp[k] for k in ("src", "d_rank", "d_row", "n_a", "n_b",
                                                                       "rot_a", "rot_b"))
        seq_a = bufs.push_async(0, x, src, None, n_a, d_rank, d_row, "rows", st.cap, n, rotate=rot_a)
        main = torch.cuda.current_stream()
        side = bufs.side_stream
        side.wait_stream(main)
        with torch.cuda.stream(side):
            seq_b = bufs.push_async(1, x, src.flip(0), None, n_b, d_rank.flip(0), d_row.flip(0), "rows", st.cap, n,
                                    rotate=rot_b)
        for t in (src, d_rank, d_row, n_b, rot_b):
            t.record_stream(side)
        bufs.wait(seq_a)
    rows = bufs.local["rows"]
    two_i = w_up.shape[2]
    s = torch.empty_strided((st.cap, two_i // 2), (_padded_cols(two_i // 2), 1), dtype=rows.dtype, device=rows.device)
    aux = torch.empty_strided((st.cap, two_i), (_padded_cols(two_i), 1), dtype=rows.dtype, device=rows.device)
    with timed("up_swiglu_fwd"):
        torch.ops.grouped_mm.swiglu_range_into(rows, w_up[:h], offs[:h], b_up[:h], aux, s, st.alpha, st.limit,
                                               True, 0)
        bufs.wait(seq_b)
        torch.ops.grouped_mm.swiglu_range_into(rows, w_up, offs, b_up, aux, s, st.alpha, st.limit, True, h)
    main.wait_stream(side)
    return s, aux


def _pipelined_combine_bwd_down(g, scale, s, w_down, aux, st):
    """Backward counterpart of _pipelined_dispatch_up: push the output gradient rows bound for every
    owner's first expert half (main stream) and the rest (side stream), run the down-proj weight + bias
    gradient and the dgrad + SwiGLU backward over experts [0, h) while the second half lands, then
    over [h, e_local) (group_begin) into the same outputs."""
    bufs, plan = st.bufs, st.plan
    offs = plan["offs"]
    sp = _split_halves(st)
    h = sp["h"]
    perm = sp["perm"]
    sc = scale[perm] if scale is not None else None
    main = torch.cuda.current_stream()
    side = bufs.side_stream
    with timed("ep_peer_combine_bwd"):
        seq_a = bufs.push_async(2, g, sp["src"], sc, sp["n_a"], sp["d_rank"], sp["d_row"], "grows", st.cap, st.n,
                                rotate=sp["rot_a"])
        side.wait_stream(main)
        with torch.cuda.stream(side):
            sc_b = sc.flip(0) if sc is not None else None
            src_b, dr_b, drow_b = sp["src"].flip(0), sp["d_rank"].flip(0), sp["d_row"].flip(0)
            seq_b = bufs.push_async(3, g, src_b, sc_b, sp["n_b"], dr_b, drow_b, "grows", st.cap, st.n,
                                    rotate=sp["rot_b"])
        g.record_stream(side)
        bufs.wait(seq_a)
    grows = bufs.local["grows"]
    el, i_dim, h_dim = w_down.shape
    dev, dt = grows.device, grows.dtype
    g_wd = torch.empty_strided((el, i_dim, h_dim), (i_dim * _padded_cols(h_dim), _padded_cols(h_dim), 1), dtype=dt,
                               device=dev)
    g_bd = torch.empty((el, h_dim), dtype=dt, device=dev)
    grad_aux = torch.empty_strided(aux.shape, (_padded_cols(aux.shape[1]), 1), dtype=dt, device=dev)
    s_t = s.transpose(-2, -1)
    w_t = w_down.transpose(-2, -1)
    with timed("down_wgrad_bias"):
        torch.ops.grouped_mm.wgrad_bias_into(s_t, grows, offs[:h], g_wd[:h], g_bd[:h], 0)
    with timed("down_dgrad_swiglu_bwd"):
        torch.ops.grouped_mm.swiglu_bwd_range_into(grows, w_t[:h], offs[:h], aux, grad_aux, st.alpha, st.limit, 0)
    bufs.wait(seq_b)
    with timed("down_wgrad_bias"):
        torch.ops.grouped_mm.wgrad_bias_into(s_t, grows, offs, g_wd, g_bd, h)
    with timed("down_dgrad_swiglu_bwd"):
        torch.ops.grouped_mm.swiglu_bwd_range_into(grows, w_t, offs, aux, grad_aux, st.alpha, st.limit, h)
    main.wait_stream(side)
    return g_wd, g_bd, grad_aux


def _padded_cols(n: int) -> int:
    return (n + 7) // 8 * 8


class _PeerMoE(torch.autograd.Function):
    """The expert-parallel MoE FFN of the peer transport in one autograd function, with the combine
    and the dispatch gradient fused into GEMM epilogues.

    forward:  push x's routed copies into the owners' `rows` (+ completion flags) -> up-proj + bias +
              SwiGLU -> down-proj + bias whose epilogue stores every output row straight into its
              source rank's `ret` buffer (mgf_gemm_desc.d_row_ptrs, NVLink peer stores) -> signal ->
              wait -> per-token weighted sum of the k returned rows.
    backward: push the output gradient (scaled by the router weights) into the owners' `grows` ->
              down-proj weight + bias gradient -> down-proj dgrad + SwiGLU backward -> up-proj dgrad
              whose epilogue stores each row's gradient into its source's `gret` -> signal -> up-proj
              weight + bias gradient (the transfer lands meanwhile) -> wait -> per-token sum of the k
              gradient rows.
    Two of the four row transfers per step thus ride inside GEMMs instead of separate pushes."""

    @staticmethod
    def forward(ctx, x, w_up, b_up, w_down, b_down, w_flat, st):
        bufs, plan = st.bufs, st.plan
        offs = plan["offs"]
        rows = bufs.local["rows"]
        el = offs.numel()
        if st.pipeline and el >= 2:
            s, aux = _pipelined_dispatch_up(x.contiguous(), w_up, b_up, st)
        else:
            with timed("ep_peer_dispatch"):
                bufs.push(0, x.contiguous(), st.copy_token, None, None, plan["dst_rank"], plan["dst_row"], "rows",
                          st.cap, st.n)
            with timed("up_swiglu_fwd"):
                s, aux = torch.ops.grouped_mm.mm_swiglu(rows, w_up, offs, b_up, st.alpha, st.limit)
        with timed("down_fwd"):
            torch.ops.grouped_mm.mm_scatter(s, w_down, offs, b_down, plan["ptr_ret"])
        bufs.wait(bufs.signal())
        with timed("ep_combine"):
            out = torch.ops.grouped_mm.combine_rows(bufs.local["ret"], st.inv_order, w_flat, st.k)
        ctx.save_for_backward(w_up, w_down, s, aux)
        ctx.w_flat, ctx.st = w_flat, st
        return out

    @staticmethod
    def backward(ctx, g):
        w_up, w_down, s, aux = ctx.saved_tensors
        st, w_flat = ctx.st, ctx.w_flat
        bufs, plan = st.bufs, st.plan
        offs = plan["offs"]
        g = g.contiguous()
        scale = w_flat[st.order].contiguous() if w_flat is not None else None
        grows = bufs.local["grows"]
        if st.pipeline and offs.numel() >= 2:
            g_wd, g_bd, grad_aux = _pipelined_combine_bwd_down(g, scale, s, w_down, aux, st)
        else:
            with timed("ep_peer_combine_bwd"):
                bufs.push(2, g, st.copy_token, scale, None, plan["dst_rank"], plan["dst_row"], "grows", st.cap, st.n)
            with timed("down_wgrad_bias"):
                g_wd, g_bd = torch.ops.grouped_mm.mm_wgrad_bias(s.transpose(-2, -1), grows, offs)
            with timed("down_dgrad_swiglu_bwd"):
                grad_aux = torch.ops.grouped_mm.mm_swiglu_bwd(grows, w_down.transpose(-2, -1), offs, aux, st.alpha,
                                                              st.limit)
        with timed("up_dgrad"):
            torch.ops.grouped_mm.mm_scatter(grad_aux, w_up.transpose(-2, -1), offs, None, plan["ptr_gret"])
        seq = bufs.signal()
        with timed("up_wgrad_bias"):
            g_wu, g_bu = torch.ops.grouped_mm.mm_wgrad_bias(bufs.local["rows"].transpose(-2, -1), grad_aux, offs)
        bufs.wait(seq)
        with timed("ep_combine"):
            gx = torch.ops.grouped_mm.combine_rows(bufs.local["gret"], st.inv_order, None, st.k)
        grad_w = None
        if w_flat is not None and ctx.needs_input_grad[5]:
            copies = bufs.local["ret"][st.inv_order].float().view(-1, st.k, g.shape[1])
            grad_w = (copies * g.float().unsqueeze(1)).sum(-1).reshape(-1)
        return gx, g_wu, g_bu.to(w_up.dtype), g_wd, g_bd.to(w_down.dtype), grad_w, None


def ep_moe_ffn_peer(x: torch.Tensor, expert_idx: torch.Tensor, num_experts: int, expert_fn: Callable,
                    bufs_cache: dict, group=None, router_weights: torch.Tensor | None = None,
                    overlap: bool = False, capacity_factor: float = 2.0, fused: dict | None = None) -> tuple:
    """Expert-parallel MoE FFN with dispatch/combine as peer-memory pushes (CUDA, world > 1).

    Same contract as ep_moe_ffn.  Every rank must pass the same number of tokens.  Each rank can
    receive at most ceil(capacity_factor * T * k) token copies (at most T * k * world); copies past
    that are dropped and MGF_DEV_ROW_OUT_OF_RANGE / MGF_DEV_BAD_OFFS are recorded in the device status
    word, which check_device_status() turns into a RuntimeError.  The receive buffers of one call stay
    live until its backward ran; a second forward before that backward raises.

    fused: {"w_up", "b_up", "w_down", "b_down", "alpha", "limit"} runs the local experts as _PeerMoE
    (combine and dispatch gradient inside the GEMM epilogues; `expert_fn` and `overlap` unused);
    None runs `expert_fn` between separate dispatch / combine pushes.
    """
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if num_experts % world:
        raise RuntimeError(f"num_experts ({num_experts}) must be divisible by the world size ({world})")
    T, H = x.shape
    k = expert_idx.shape[1]
    e_local = num_experts // world
    n = T * k
    cap = min(n * world, int(math.ceil(capacity_factor * n)))
    cap = (cap + 7) // 8 * 8
    key = (n, cap, H, x.dtype)
    bufs = bufs_cache.get(key)
    if bufs is None:
        bufs = PeerBuffers({"rows": (cap, H), "grows": (cap, H), "ret": (n, H), "gret": (n, H)}, x.dtype, x.device,
                           group)
        bufs_cache.clear()
        bufs_cache[key] = bufs
    if getattr(bufs, "pending_backward", False) and torch.is_grad_enabled():
        raise RuntimeError("ep_moe_ffn_peer: a second forward before the previous one's backward would overwrite "
                           "its receive buffers")
    st = _PeerState()
    with timed("ep_plan"):
        order, inv_order, copy_token, e_sorted, counts = torch.ops.grouped_mm.ep_sort(expert_idx, num_experts, k)
        st.order, st.inv_order, st.copy_token, st.e_sorted = order, inv_order, copy_token, e_sorted
        c_all = torch.empty(world, num_experts, dtype=counts.dtype, device=x.device)
        # the count exchange also orders this call after every rank's previous use of the buffers
        dist.all_gather_into_tensor(c_all, counts, group=group)
        r = torch.ops.grouped_mm.ep_routes(c_all, e_sorted, rank, cap, bufs.bases["ret"], bufs.bases["gret"],
                                           H * x.element_size())
        st.plan = {"dst_rank": r[0], "dst_row": r[1], "src_rank": r[2], "src_pos": r[3], "offs": r[4],
                   "n_recv": r[5], "ptr_ret": r[6], "ptr_gret": r[7]}
    st.bufs, st.k, st.n, st.cap = bufs, k, n, cap
    st.side_stream = bufs.side_stream
    st.dispatch_bwd_done = None
    st.overlap = overlap
    if fused is not None:
        st.alpha, st.limit = fused["alpha"], fused["limit"]
        st.pipeline = fused.get("pipeline", False)
        w_flat = router_weights.reshape(-1).float().contiguous() if router_weights is not None else None
        out = _PeerMoE.apply(x, fused["w_up"], fused["b_up"], fused["w_down"], fused["b_down"], w_flat, st)
        bufs.pending_backward = out.requires_grad
        if out.requires_grad:
            out.register_hook(lambda g: (setattr(bufs, "pending_backward", False), g)[1])
        return out, st
    rows = _PeerDispatch.apply(x, st)
    y = expert_fn(rows, st.plan["offs"], st) if getattr(expert_fn, "takes_peer_state", False) else \
        expert_fn(rows, st.plan["offs"])
    w_flat = router_weights.reshape(-1).float().contiguous() if router_weights is not None else None
    out = _PeerCombine.apply(y, w_flat, st)
    bufs.pending_backward = out.requires_grad
    if out.requires_grad:
        out.register_hook(lambda g: (setattr(bufs, "pending_backward", False), g)[1])
    return out, st


class EPMoEFFN(torch.nn.Module):
    """GPT-OSS-style MoE FFN whose E experts are sharded E/N per rank, run with the fused kernels."""

    def __init__(self, num_experts: int, hidden: int, inter: int, group=None, device=None, seed: int = 0,
                 swiglu_alpha: float = 1.702, swiglu_limit: float = 7.0, transport: str = "peer",
                 overlap: bool = False, capacity_factor: float = 2.0, fused: bool = True,
                 pipeline: bool = False):
        """transport: "peer" (NVLink pushes, CUDA, world > 1) or "nccl" (all-to-all).  overlap (peer
        transport): push the dispatch's gradient on a side stream under the up-projection weight
        gradient instead of after it.  capacity_factor (peer transport): receive buffers hold
        ceil(capacity_factor * tokens * topk) rows per rank (overflow is reported, see
        ep_moe_ffn_peer).  fused (peer transport): the combine and the dispatch gradient are written by
        the down-proj forward / up-proj dgrad epilogues straight into the source ranks (_PeerMoE);
        False: separate push kernels around the FFN (then `overlap` applies).  pipeline (fused peer
        transport, at least 2 local experts): the dispatch and the up-projection run in two halves
        of the local experts, the second half's push overlapping the first half's GEMM (and the
        combine-gradient push likewise with the down-proj backward); off by default since the
        second tail wave of each split GEMM costs about what the overlap saves."""
        super().__init__()
        self.fused = fused
        self.pipeline = pipeline
        self.overlap = overlap
        self.capacity_factor = capacity_factor
        if transport not in ("peer", "nccl"):
            raise ValueError(f"transport must be 'peer' or 'nccl', got {transport!r}")
        self.transport = transport
        self._peer_bufs: dict = {}
        from .workloads import MoEShape, make_weights_device

        world = dist.get_world_size(group) if dist.is_initialized() else 1
        rank = dist.get_rank(group) if dist.is_initialized() else 0
        if num_experts % world:
            raise RuntimeError(f"num_experts ({num_experts}) must be divisible by the world size ({world})")
        self.num_experts, self.group = num_experts, group
        self.e_local = num_experts // world
        self.alpha, self.limit = swiglu_alpha, swiglu_limit
        w_up, b_up, w_down, b_down = make_weights_device(MoEShape(self.e_local, hidden, inter),
                                                         seed=seed + 7919 * rank, device=device)
        self.w_up = torch.nn.Parameter(w_up)
        self.b_up = torch.nn.Parameter(b_up)
        self.w_down = torch.nn.Parameter(w_down)
        self.b_down = torch.nn.Parameter(b_down)
        self.last_local_rows = 0

    def expert_fn(self, rows: torch.Tensor, offs: torch.Tensor) -> torch.Tensor:
        from . import grouped_mm_downproj, grouped_mm_swiglu

        s, aux = grouped_mm_swiglu(rows, self.w_up, offs, self.b_up, self.alpha, self.limit)
        return grouped_mm_downproj(s, self.w_down, offs, self.b_down, aux, self.alpha, self.limit)

    def _peer_expert_fn(self, rows: torch.Tensor, offs: torch.Tensor, st) -> torch.Tensor:
        return _EPExpertFFN.apply(rows, self.w_up, self.b_up, self.w_down, self.b_down, offs, self.alpha,
                                  self.limit, st)

    _peer_expert_fn.takes_peer_state = True

    def forward(self, x: torch.Tensor, expert_idx: torch.Tensor, router_weights: torch.Tensor | None = None):
        world = dist.get_world_size(self.group) if dist.is_initialized() else 1
        if self.transport == "peer" and world > 1 and x.is_cuda:
            fused = None
            if self.fused:
                fused = {"w_up": self.w_up, "b_up": self.b_up, "w_down": self.w_down, "b_down": self.b_down,
                         "alpha": self.alpha, "limit": self.limit, "pipeline": self.pipeline}
            out, st = ep_moe_ffn_peer(x, expert_idx, self.num_experts, self._peer_expert_fn, self._peer_bufs,
                                      self.group, router_weights, overlap=self.overlap,
                                      capacity_factor=self.capacity_factor, fused=fused)
            self.last_local_rows = st.plan["n_recv"]  # device tensor; read it outside timed regions
            return out
        out, plan = ep_moe_ffn(x, expert_idx, self.num_experts, self.expert_fn, self.group, router_weights)
        self.last_local_rows = plan.local_rows
        return out
