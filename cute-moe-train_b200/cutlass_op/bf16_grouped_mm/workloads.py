"""Seeded synthetic MoE FFN workloads with the shapes and value distributions of the benchmark
configurations (no dataset is involved).

* config 1: E=8, H=2048, I=1024, tokens_per_expert [128,64,0,256,192,32,128,64] (M=864), seed 0
  -- the reference README's quick-start shapes (README.md:44-56).
* config 2/3: GPT-OSS-20B expert shape E=32, H=I=2880, 24576 tokens, top-4 (M=98304), experts per
  token drawn without replacement from Zipf(s=1.1) over a seeded expert permutation; config 3
  forces >= 2 experts to receive no tokens.
* config 4: GPT-OSS-120B expert shape E=128, H=I=2880, top-4, 24576 tokens per rank.
* config 5: E=256, H=7168, I=2048, top-8, Zipf(s=1.3) plus forced group sizes 0, 1, 7 and 129.

Values: x ~ N(0,1); W ~ N(0,1)/sqrt(fan_in); biases ~ N(0, 0.02); all rounded to bf16.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch


@dataclass
class MoEShape:
    E: int
    H: int
    I: int


CONFIG1_TPE = [128, 64, 0, 256, 192, 32, 128, 64]


def zipf_routing(tokens: int, E: int, topk: int, s: float, seed: int, zero_experts: int = 0,
                 device: str | torch.device = "cpu") -> torch.Tensor:
    """Tokens per expert for `tokens` tokens routed top-`topk` without replacement.

    Expert popularity follows Zipf(s) over a seeded permutation of the experts (Gumbel top-k
    sampling draws k distinct experts per token with those weights).  The `zero_experts` least
    popular experts get no tokens at all.
    """
    g = torch.Generator(device="cpu").manual_seed(seed)
    perm = torch.randperm(E, generator=g)
    ranks = torch.arange(1, E + 1, dtype=torch.float64)
    w = ranks.pow(-s)
    if zero_experts:
        w[E - zero_experts:] = 0.0
    weights = torch.zeros(E, dtype=torch.float64)
    weights[perm] = w
    logw = torch.log(weights).float()
    counts = torch.zeros(E, dtype=torch.int64)
    chunk = 8192
    for start in range(0, tokens, chunk):
        n = min(chunk, tokens - start)
        u = torch.rand(n, E, generator=g).clamp_(1e-12, 1.0 - 1e-7)
        keys = logw.unsqueeze(0) - torch.log(-torch.log(u))
        top = keys.topk(topk, dim=1).indices
        counts += torch.bincount(top.flatten(), minlength=E)
    return counts.to(device)


def force_group_sizes(counts: torch.Tensor, sizes=(0, 1, 7, 129), seed: int = 0) -> torch.Tensor:
    """Config 5's forced ragged groups: give len(sizes) seeded experts (never the largest) exactly
    those token counts, keeping the total: the surplus goes to the largest expert, a deficit is taken
    from the largest experts in turn (never below zero)."""
    counts = counts.clone()
    g = torch.Generator(device="cpu").manual_seed(seed + 17)
    big = int(torch.argmax(counts))
    cand = [int(e) for e in torch.randperm(counts.numel(), generator=g) if int(e) != big][: len(sizes)]
    delta = 0
    for e, sz in zip(cand, sizes):
        delta += int(counts[e]) - sz
        counts[e] = sz
    if delta >= 0:
        counts[big] += delta
    else:
        need = -delta
        for e in torch.argsort(counts, descending=True).tolist():
            if e in cand:
                continue
            take = min(need, int(counts[e]))
            counts[e] -= take
            need -= take
            if need == 0:
                break
        if need:
            raise ValueError("force_group_sizes: not enough tokens to force the requested group sizes")
    return counts


def config5_counts(tokens: int, E: int = 256, topk: int = 8, seed: int = 0) -> torch.Tensor:
    """Config 5 routing: top-8 of Zipf(1.3) over 256 experts, then forced groups of 0, 1, 7 and 129."""
    return force_group_sizes(zipf_routing(tokens, E, topk, 1.3, seed=seed), seed=seed)


def offs_from_counts(counts: torch.Tensor) -> torch.Tensor:
    return torch.cumsum(counts.to(torch.int64), 0).to(torch.int32)


def make_weights(shape: MoEShape, seed: int, device="cpu", dtype=torch.bfloat16):
    """(W_up [E,H,2I], b_up [E,2I], W_down [E,I,H], b_down [E,H]) with the spec's distributions."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    E, H, I = shape.E, shape.H, shape.I
    w_up = (torch.randn(E, H, 2 * I, generator=g) / math.sqrt(H)).to(dtype)
    b_up = (torch.randn(E, 2 * I, generator=g) * 0.02).to(dtype)
    w_down = (torch.randn(E, I, H, generator=g) / math.sqrt(I)).to(dtype)
    b_down = (torch.randn(E, H, generator=g) * 0.02).to(dtype)
    return w_up.to(device), b_up.to(device), w_down.to(device), b_down.to(device)


def make_weights_device(shape: MoEShape, seed: int, device, dtype=torch.bfloat16):
    """Like make_weights but drawn on the device (large shapes; a different stream of numbers)."""
    g = torch.Generator(device=device).manual_seed(seed)
    E, H, I = shape.E, shape.H, shape.I
    w_up = (torch.randn(E, H, 2 * I, generator=g, device=device) / math.sqrt(H)).to(dtype)
    b_up = (torch.randn(E, 2 * I, generator=g, device=device) * 0.02).to(dtype)
    w_down = (torch.randn(E, I, H, generator=g, device=device) / math.sqrt(I)).to(dtype)
    b_down = (torch.randn(E, H, generator=g, device=device) * 0.02).to(dtype)
    return w_up, b_up, w_down, b_down


def config1(device="cpu"):
    """Config 1 (E=8, H=2048, I=1024, the reference quick-start token counts), generated in the
    order x, W_up, b_up, W_down, b_down from seed 0."""
    E, H, I = 8, 2048, 1024
    g = torch.Generator(device="cpu").manual_seed(0)
    counts = torch.tensor(CONFIG1_TPE, dtype=torch.int64)
    M = int(counts.sum())
    x = torch.randn(M, H, generator=g).to(torch.bfloat16)
    w_up = (torch.randn(E, H, 2 * I, generator=g) / math.sqrt(H)).to(torch.bfloat16)
    b_up = (torch.randn(E, 2 * I, generator=g) * 0.02).to(torch.bfloat16)
    w_down = (torch.randn(E, I, H, generator=g) / math.sqrt(I)).to(torch.bfloat16)
    b_down = (torch.randn(E, H, generator=g) * 0.02).to(torch.bfloat16)
    offs = offs_from_counts(counts)
    t = [x, w_up, b_up, w_down, b_down, offs]
    return [v.to(device) for v in t]


def small_case(E: int, H: int, I: int, counts: list[int], seed: int, device="cpu", grad: str = "randn"):
    """A small seeded case: (x, W_up, b_up, W_down, b_down, offs, grad_out)."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    M = int(sum(counts))
    x = torch.randn(M, H, generator=g).to(torch.bfloat16)
    w_up = (torch.randn(E, H, 2 * I, generator=g) / math.sqrt(H)).to(torch.bfloat16)
    b_up = (torch.randn(E, 2 * I, generator=g) * 0.02).to(torch.bfloat16)
    w_down = (torch.randn(E, I, H, generator=g) / math.sqrt(I)).to(torch.bfloat16)
    b_down = (torch.randn(E, H, generator=g) * 0.02).to(torch.bfloat16)
    if grad == "ones":
        gout = torch.ones(M, H).to(torch.bfloat16)
    else:
        gout = torch.randn(M, H, generator=g).to(torch.bfloat16)
    offs = offs_from_counts(torch.tensor(counts, dtype=torch.int64))
    return [v.to(device) for v in (x, w_up, b_up, w_down, b_down, offs, gout)]


def ffn_flops(M: int, H: int, I: int, backward: bool = True) -> float:
    """Useful FLOPs: forward 6*M*H*I (up 4MHI + down 2MHI); forward+backward 18*M*H*I."""
    return (18.0 if backward else 6.0) * M * H * I
