#!/usr/bin/env python
"""Benchmark of the MoE FFN grouped-GEMM path on B200.

Metric: MoE FFN fwd+bwd ms and BF16 TFLOP/s per GPU (24K tokens per rank), % of
tensor peak.  One step = grouped_mm_swiglu -> grouped_mm_downproj -> out.sum().backward() over the
routed rows of 24576 tokens (top-4): useful FLOPs 18*M*H*I (M = routed rows on this GPU).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload ...]

N=1 runs config 3 (GPT-OSS-20B experts, E=32, H=I=2880, Zipf(1.1) top-4 routing with two experts
receiving no tokens).  N>1 (torchrun) runs config 4 under expert parallelism (GPT-OSS-120B experts,
E=128 split E/N per GPU, 24576 tokens per rank, NVLink peer-memory dispatch/combine), weak scaling,
after an expert-parallel parity self-check against the oracle (``ep_parity``).  At N=1 the line also
carries secondary measurements (``extra``: cfg2 forward, cfg5 at 4096 tokens, the FP8 FFN, cfg4 on one
GPU), the torch._grouped_mm comparator, the end-to-end leg and the CPU baseline.
``--impl reference`` times the reference's own Python layer over a CPU restatement of its kernels.
All inputs are seeded synthetic data of the configured shapes.  Rank 0 prints one JSON line.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import tempfile
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
PKG = REPO / "cute-moe-train_b200"
for _p in (str(REPO), str(PKG)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "MoE FFN fwd+bwd ms & BF16 TFLOP/s per GPU (24K tok/rank), % of tensor peak"
UNIT = "TFLOP/s"
ALPHA, LIMIT = 1.702, 7.0
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

# FLOPs of each operator per launch, in units of M*H*I (M routed rows on this GPU).
OP_FLOP_UNITS = {
    "up_swiglu_fwd": 4, "down_fwd": 2, "down_wgrad_bias": 2, "down_dgrad_swiglu_bwd": 2,
    "up_dgrad": 4, "up_wgrad_bias": 4, "up_recompute_aux": 4, "fp8_up_swiglu_fwd": 4,
}


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=60)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["auto", "cfg2", "cfg3", "cfg4", "cfg5"], default="auto",
                    help="cfg3 (1 GPU) / cfg4 (EP) by default; cfg2 = forward only; cfg5 = E=256 fine-grained")
    ap.add_argument("--routing", choices=["zipf", "uniform"], default="uniform",
                    help="expert-parallel routing (cfg4 lists both; uniform is the balanced case)")
    ap.add_argument("--ep-overlap", action="store_true",
                    help="peer transport: push the dispatch gradient under the up-proj weight gradient")
    ap.add_argument("--ep-unfused", action="store_true",
                    help="peer transport: separate push kernels for the combine and the dispatch gradient instead "
                         "of the GEMM scatter epilogues")
    ap.add_argument("--ep-pipeline", action="store_true",
                    help="peer transport: the dispatch / combine-gradient pushes pipelined with the GEMMs in two "
                         "expert halves (measured neutral to 1% slower at 8 GPUs, so off by default)")
    ap.add_argument("--transport", choices=["peer", "nccl"], default="peer",
                    help="expert-parallel dispatch/combine: peer-memory pushes or NCCL all-to-all")
    ap.add_argument("--no-compare", action="store_true", help="skip the torch._grouped_mm comparator")
    ap.add_argument("--fp8", action="store_true",
                    help="cfg2 only: the e4m3 up-projection + SwiGLU (row-wise scales; inputs quantised "
                         "before the timed region)")
    ap.add_argument("--recompute-aux", action="store_true",
                    help="store_aux=False: the forward keeps no aux, the backward recomputes it "
                         "(the extra GEMM's FLOPs are not counted in the metric)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--cpu-baseline-only", action="store_true", help=argparse.SUPPRESS)
    ap.add_argument("--no-extra", action="store_true",
                    help="N=1: skip the secondary measurements (cfg2 forward, cfg5 at 4096 tokens, cfg4 at N=1)")
    ap.add_argument("--tokens", type=int, default=0,
                    help="tokens per GPU (default 24576; cfg5 default 4096; smaller for profiling cases)")
    ap.add_argument("--experts", type=int, default=0, help="override the number of experts (profiling cases)")
    return ap.parse_args()


def load_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {k: float(d[k]) for k in ("hbm_gbs", "bf16_tflops", "bf16_tflops_sustained")}, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def load_traffic():
    """Per-launch DRAM bytes of each launch of the step from the committed ncu summary, if any."""
    p = REPO / "profiles" / "launch_traffic_cfg3.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except Exception:
            return None
    return None


# ------------------------------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi clock / throttle-reason samples every 200 ms while the timed region runs."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.gpu_id, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) == 8:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        def num(v):
            try:
                return float(v)
            except ValueError:
                return None

        sm = sorted(v for v in (num(r[0]) for r in rows) if v is not None)
        power = [v for v in (num(r[2]) for r in rows) if v is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[4 + i].strip().lower() == "active"})
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": num(rows[0][1]),
                "reasons": reasons, "samples": len(rows), "power_w_max": max(power) if power else None}


# ------------------------------------------------------------------------------------- workload

def build_workload(args, rank, world, device):
    """(name, description, E, forced-empty experts, tokens, top-k, H, I, zipf s, forward only)."""
    wl = args.workload if args.workload != "auto" else ("cfg3" if world == 1 else "cfg4")
    if wl == "cfg5":
        tokens = args.tokens or 4096
        E_total = args.experts or 256
        desc = (f"cfg5: fine-grained E={E_total} H=7168 I=2048, {tokens} tokens top-8 Zipf(1.3) with forced "
                f"groups of 0, 1, 7 and 129 rows, fwd+bwd")
        return wl, desc, E_total, 0, tokens, 8, 7168, 2048, 1.3, False
    tokens, topk, H, I = args.tokens or 24576, 4, 2880, 2880
    if wl in ("cfg2", "cfg3"):
        E_total = args.experts or 32
        zero = 2 if wl == "cfg3" else 0
        if wl == "cfg3":
            desc = (f"cfg3: GPT-OSS-20B experts E={E_total} H=I=2880, {tokens} tokens top-4 Zipf(1.1), "
                    f"2 experts with 0 tokens")
        else:
            desc = f"cfg2: forward-only grouped_mm_swiglu, E={E_total} H=I=2880, {tokens} tokens top-4 Zipf(1.1)"
        return wl, desc, E_total, zero, tokens, topk, H, I, 1.1, wl == "cfg2"
    E_total = args.experts or 128
    desc = (f"cfg4: GPT-OSS-120B experts E={E_total} H=I=2880, {tokens} tokens/rank top-4 {args.routing} routing, "
            f"expert parallel E/{world} per GPU, dispatch/combine by "
            + (("peer-memory pushes over NVLink" + ("" if args.ep_unfused else
                                                     ", combine and dispatch gradient stored by the GEMM epilogues"
                                                     + ("" if not args.ep_pipeline else
                                                        ", pushes pipelined with the GEMMs in two expert halves")))
               if args.transport == "peer" else "NCCL all-to-all")
            + (", dispatch gradient pushed under the up-proj wgrad" if args.ep_overlap else ""))
    return wl, desc, E_total, 0, tokens, topk, H, I, 1.1, False


def line_config(args, world):
    """The `config` object of the JSON line: identical for this arm and the reference arm."""
    wl, desc, E_total, _, tokens, topk, H, I, _, fwd_only = build_workload(args, 0, world, None)
    return {"workload": desc, "E": E_total, "H": H, "I": I, "tokens_per_gpu": tokens, "topk": topk,
            "parallelism": f"ep{world}" if world > 1 else "single",
            "l2": "inputs larger than L2 (x 566 MB + weights >= 1.6 GB per GPU), no flush",
            "step": (("grouped_mm_swiglu_fp8 forward only (config 2 shapes, row-wise e4m3 inputs "
                      "quantised before the timed region)" if args.fp8 else
                      "grouped_mm_swiglu forward only (config 2)") if fwd_only else
                     "grouped_mm_swiglu -> grouped_mm_downproj -> out.sum().backward(); no optimizer "
                     "(the metric is the MoE FFN fwd+bwd)"
                     + ("; store_aux=False: aux recomputed in backward, 18*M*H*I FLOPs counted"
                        if args.recompute_aux else ""))}


def load_workloads_module():
    """workloads.py by file path: the seeded generators without importing the product package
    (whose __init__ loads the native libraries)."""
    import importlib.util

    path = PKG / "cutlass_op" / "bf16_grouped_mm" / "workloads.py"
    if "mgf_bench_workloads" in sys.modules:
        return sys.modules["mgf_bench_workloads"]
    spec = importlib.util.spec_from_file_location("mgf_bench_workloads", path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules["mgf_bench_workloads"] = mod  # dataclasses look their module up here
    spec.loader.exec_module(mod)
    return mod


# ------------------------------------------------------------------------------------- runs

def time_steps(step_fn, steps, warmup, barrier=None, sync=None, tail=None):
    """Device time per step.  `tail` runs after the last step, inside the timed window (work the
    steps issued on other streams that must be counted)."""
    import torch

    for _ in range(warmup):
        step_fn()
    torch.cuda.synchronize()
    if barrier:
        barrier()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        step_fn()
    if tail:
        tail()
    b.record()
    torch.cuda.synchronize()
    if barrier:
        barrier()
    return a.elapsed_time(b) / steps


REF_LAYER = REPO / "baseline" / "_ref" / "group_gemm"


class CpuReference:
    """The reference's CPU path for this workload, timed on the host cores.

    Preferred: the reference's own, unmodified Python layer (its __init__.py + custom_op.py staged
    under baseline/_ref by baseline/stage_reference.py: autograd routing, fused-only contract,
    _segment_sum_rows) over oracle/ref_ext_cpu.py, a CPU restatement of its three CUDA kernels
    (kind "reference").  Without the staged layer: the oracle port oracle/moe_ffn.kernel_chain
    (kind "port").  Neither loads any of this repository's native libraries."""

    def __init__(self):
        import torch

        torch.set_num_threads(os.cpu_count() or 1)
        self.cores = torch.get_num_threads()
        self.ref = None
        if (REF_LAYER / "custom_op.py").is_file():
            from oracle.ref_ext_cpu import load_reference_layer

            self.ref = load_reference_layer(REF_LAYER, modname="ref_group_gemm")
            self.kind = "reference"
            self.what = ("the reference's unmodified Python layer (baseline/_ref/group_gemm: __init__.py + "
                         "custom_op.py) over a CPU restatement of its three CUDA kernels (oracle/ref_ext_cpu.py), "
                         "torch fp32 GEMMs on bf16 inputs")
        else:
            self.kind = "port"
            self.what = "the oracle port (oracle/moe_ffn.kernel_chain, fp32 torch CPU restatement of the chain)"

    def step(self, case):
        x, w_up, b_up, w_down, b_down, offs = case
        if self.ref is None:
            from oracle import moe_ffn as O

            g = __import__("torch").ones(x.shape[0], w_down.shape[-1], dtype=x.dtype)
            O.kernel_chain(x, w_up, b_up, w_down, b_down, offs, g)
            return
        leaves = [t.detach().requires_grad_(True) for t in (x, w_up, b_up, w_down, b_down)]
        xl, wu, bu, wd, bd = leaves
        s_, aux = self.ref.grouped_mm_swiglu(xl, wu, offs=offs, bias=bu, swiglu_alpha=ALPHA, swiglu_limit=LIMIT)
        out = self.ref.grouped_mm_downproj(s_, wd, offs=offs, bias=bd, aux_biased_acc=aux, swiglu_alpha=ALPHA,
                                           swiglu_limit=LIMIT)
        out.sum().backward()


def cpu_counts(args, world):
    """Tokens per local expert of rank 0's workload (the same routing the GPU arm uses)."""
    import torch

    wlm = load_workloads_module()
    wl, _, E_total, zero, tokens, topk, H, I, zipf_s, fwd_only = build_workload(args, 0, world, None)
    if world == 1:
        if wl == "cfg5":
            return wlm.config5_counts(tokens, E_total, topk, seed=0), H, I, fwd_only
        return wlm.zipf_routing(tokens, E_total, topk, zipf_s, seed=0, zero_experts=zero), H, I, fwd_only
    # expert parallel: rank 0 owns E/N experts and receives ~tokens*topk rows from all ranks
    e_local = E_total // world
    rows = tokens * topk
    c = torch.full((e_local,), rows // e_local, dtype=torch.int64)
    c[: rows % e_local] += 1
    return c, H, I, fwd_only


def cpu_case(counts, H, I, seed=123):
    import math

    import torch

    g = torch.Generator().manual_seed(seed)
    E, M = counts.numel(), int(counts.sum())
    x = torch.randn(M, H, generator=g).to(torch.bfloat16)
    w_up = (torch.randn(E, H, 2 * I, generator=g) / math.sqrt(H)).to(torch.bfloat16)
    b_up = (torch.randn(E, 2 * I, generator=g) * 0.02).to(torch.bfloat16)
    w_down = (torch.randn(E, I, H, generator=g) / math.sqrt(I)).to(torch.bfloat16)
    b_down = (torch.randn(E, H, generator=g) * 0.02).to(torch.bfloat16)
    offs = torch.cumsum(counts, 0).to(torch.int32)
    return x, w_up, b_up, w_down, b_down, offs


def cpu_sample_tflops(args, world, target_s=12.0):
    """cpu_baseline of this arm's line: the CPU reference on a bounded sample of the workload -- the
    first experts of its routing, whole, up to about an eighth of the rows -- one untimed run, then
    repeated until about target_s seconds of CPU work were timed."""
    cref = CpuReference()
    counts, H, I, _ = cpu_counts(args, world)
    keep, rows = 0, 0
    for c in counts.tolist():
        if rows >= max(1, int(counts.sum()) // 8):
            break
        keep += 1
        rows += c
    case = cpu_case(counts[:keep], H, I)
    cref.step(case)
    reps, total = 0, 0.0
    while total < target_s and reps < 20:
        t0 = time.perf_counter()
        cref.step(case)
        total += time.perf_counter() - t0
        reps += 1
    value = 18.0 * rows * H * I * reps / total / 1e12
    sample = (f"{cref.what}: fwd+bwd of the first {keep} of {counts.numel()} experts of this workload's routing "
              f"({rows} routed rows, H={H}, I={I}), one untimed run then {reps} timed, {total:.1f} s of CPU work")
    return {"value": value, "unit": UNIT, "cores": cref.cores, "kind": cref.kind, "sample": sample}


def cpu_baseline_subprocess(args):
    """cpu_sample_tflops in a child process: the reference layer registers the same `grouped_mm`
    operator namespace as this repository's native library, so it cannot share this process."""
    cmd = [sys.executable, str(Path(__file__).resolve()), "--cpu-baseline-only", "--workload", args.workload]
    if args.tokens:
        cmd += ["--tokens", str(args.tokens)]
    if args.experts:
        cmd += ["--experts", str(args.experts)]
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=900, env=dict(os.environ, **MALLOC_ENV))
        lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
        if r.returncode == 0 and lines:
            return json.loads(lines[-1])
        return {"error": f"rc={r.returncode}: {r.stderr[-300:]}"}
    except Exception as e:
        return {"error": f"{type(e).__name__}: {str(e)[:200]}"}


def reference_arm(args, rank, world):
    """--impl reference: the reference's CPU path (CpuReference) on this arm's workload and config,
    timed on the host cores.  Each step runs the whole workload of rank 0 when K + W such steps fit
    in REF_BUDGET_S seconds; otherwise each step is a bounded sample of it -- the first experts of
    its routing, whole -- sized from a calibration step so that the run fits (stated in the line)."""
    if rank != 0:
        return
    cref = CpuReference()
    counts, H, I, fwd_only = cpu_counts(args, world)
    if fwd_only:
        raise SystemExit("--impl reference times the fwd+bwd workloads (cfg3/cfg4/cfg5)")
    total_rows = int(counts.sum())
    # calibration on about an eighth of the experts
    n_cal = max(1, counts.numel() // 8)
    cal = cpu_case(counts[:n_cal], H, I)
    cref.step(cal)
    t0 = time.perf_counter()
    cref.step(cal)
    t_cal = time.perf_counter() - t0
    rows_cal = max(1, int(counts[:n_cal].sum()))
    per_row = t_cal / rows_cal
    allowed = REF_BUDGET_S / max(1, args.steps + args.warmup)
    keep, rows = 0, 0
    for c in counts.tolist():
        if keep and (rows + c) * per_row > allowed:
            break
        keep += 1
        rows += c
    del cal
    case = cpu_case(counts[:keep], H, I)
    for _ in range(args.warmup):
        cref.step(case)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        cref.step(case)
        times.append(time.perf_counter() - t0)
    step_s = sum(times) / len(times)
    value = 18.0 * rows * H * I / step_s / 1e12
    whole = keep == counts.numel()
    sample = (f"{cref.what}: fwd+bwd with out.sum(); every step " +
              (f"the whole workload of rank 0 ({counts.numel()} experts, {rows} routed rows" if whole else
               f"a bounded sample of rank 0's workload: its first {keep} of {counts.numel()} experts, whole "
               f"({rows} of {total_rows} routed rows; the full step would take ~{per_row * total_rows:.0f} s here")
              + f", H={H}, I={I}); malloc keeps freed memory (no page-fault churn)")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": step_s * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32 (bf16-rounded inputs)", "data": "synthetic",
        "config": line_config(args, world),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cref.cores, "kind": cref.kind, "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "rows_per_step": rows, "routed_rows_rank0": total_rows, "whole_workload_per_step": whole,
    }
    print(json.dumps(line), flush=True)


# glibc malloc settings for the CPU legs: keep freed memory in the process instead of returning each
# large block to the kernel and faulting it in again (the CPU path allocates GB-sized temporaries
# every step; without this, page faults roughly double its time).
MALLOC_ENV = {"MALLOC_MMAP_THRESHOLD_": str(16 << 30), "MALLOC_TRIM_THRESHOLD_": str(64 << 30),
              "MALLOC_TOP_PAD_": str(1 << 30)}
REF_BUDGET_S = 200.0


def _reexec_with_malloc_env():
    if all(os.environ.get(k) == v for k, v in MALLOC_ENV.items()):
        return
    env = dict(os.environ, **MALLOC_ENV)
    os.execve(sys.executable, [sys.executable] + sys.argv, env)


def ep_parity_check(args, world, rank, device):
    """Before the timed region at N > 1: a small expert-parallel fwd+bwd (512 tokens per rank, 8
    experts per rank, H=256, I=128, top-4, Zipf routing, router weights, random output gradient)
    through the same transport as the bench; rank 0 gathers every rank's inputs, weights and
    results and checks outputs, token, router-weight and all expert weight/bias gradients against
    the single-process oracle (oracle/ep_ffn.py, used here only as the checker)."""
    import torch
    import torch.distributed as dist

    from cutlass_op.bf16_grouped_mm.expert_parallel import EPMoEFFN, route_tokens

    T, E, H, I, K = 512, 8 * world, 256, 128, 4
    ffn = EPMoEFFN(E, H, I, device=device, seed=77, transport=args.transport, overlap=args.ep_overlap,
                   fused=not args.ep_unfused)
    g = torch.Generator().manual_seed(500 + rank)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    w = torch.rand(T, K, generator=g)
    gout = torch.randn(T, H, generator=g).to(torch.bfloat16)
    idx = route_tokens(T, E, K, "zipf", seed=600 + rank)
    xd, wd = x.to(device).requires_grad_(True), w.to(device).requires_grad_(True)
    out = ffn(xd, idx.to(device), wd)
    out.backward(gout.to(device))
    torch.cuda.synchronize()
    mine = {"x": x, "idx": idx, "w": w, "g": gout,
            "got": [t.detach().cpu() for t in (out, xd.grad, wd.grad, ffn.w_up.grad, ffn.b_up.grad,
                                              ffn.w_down.grad, ffn.b_down.grad)],
            "weights": [p.detach().cpu() for p in (ffn.w_up, ffn.b_up, ffn.w_down, ffn.b_down)]}
    allr = [None] * world
    dist.all_gather_object(allr, mine)
    del ffn
    if rank != 0:
        return None
    from oracle import moe_ffn as O
    from oracle.ep_ffn import ep_reference

    wts = [torch.cat([r["weights"][i] for r in allr], 0) for i in range(4)]
    want = ep_reference([r["x"] for r in allr], [r["idx"] for r in allr], [r["w"] for r in allr],
                        [r["g"] for r in allr], *wts)
    e_local = E // world
    worst_rel, worst_cos, ok, n = 0.0, 1.0, True, 0
    for rk, r in enumerate(allr):
        sl = slice(rk * e_local, (rk + 1) * e_local)
        refs = [want["out"][rk], want["dx"][rk], want["dw_router"][rk], want["dw_up"][sl], want["db_up"][sl],
                want["dw_down"][sl], want["db_down"][sl]]
        for got, ref in zip(r["got"], refs):
            c = O.check("ep", got.float(), ref.float())
            worst_rel, worst_cos, ok, n = max(worst_rel, c["rel"]), min(worst_cos, c["cos"]), ok and c["ok"], n + 1
    return {"ok": ok, "max_rel": worst_rel, "min_cos": worst_cos, "tensors_checked": n,
            "case": f"{world} ranks x {T} tokens, E={E} H={H} I={I} top-{K} Zipf, router weights, random grad, "
                    f"transport {args.transport}" + (" + overlap" if args.ep_overlap else "")}


def measure_e4m3_peak(device):
    """Burst e4m3 GEMM throughput of this GPU: cuBLAS via torch._scaled_mm, 8192^3, best of 13 (TFLOP/s)."""
    import torch

    a = torch.randn(8192, 8192, device=device).to(torch.float8_e4m3fn)
    b = torch.randn(8192, 8192, device=device).to(torch.float8_e4m3fn).t()
    one = torch.ones((), device=device)
    best = 1e9
    for _ in range(13):
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record()
        torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
        ev1.record()
        torch.cuda.synchronize()
        best = min(best, ev0.elapsed_time(ev1))
    del a, b
    torch.cuda.empty_cache()
    return 2 * 8192 ** 3 / (best * 1e-3) / 1e12


def roofline_entry(ops, local_rows, H, I, peaks, peak_src, fp8=False, steps=None, fp8_peak=None):
    """Live per-kernel roofline of the step: achieved TFLOP/s of the dominant operator (its FLOPs per
    step / its CUDA-event time per step; an operator run as several launches over expert ranges counts
    all of them) against the measured burst bf16 peak, the sustained one beside."""
    names = [k for k in ops if k in OP_FLOP_UNITS]
    if not names:
        return None

    def per_step_ms(v):
        return v["total_ms"] / steps if steps else v["avg_ms"]

    name = max(names, key=lambda k: ops[k]["total_ms"])
    fl = OP_FLOP_UNITS[name] * float(local_rows) * H * I
    ach = fl / (per_step_ms(ops[name]) * 1e-3) / 1e12
    peak, peak_name = peaks["bf16_tflops"], f"{peak_src} bf16_tflops (burst)"
    if fp8:  # the e4m3 burst measured on this GPU, else the nominal dense figure
        peak, peak_name = ((fp8_peak, "measured e4m3 burst (torch._scaled_mm 8192^3 on this GPU)") if fp8_peak else
                           (4500.0, "nominal e4m3 dense 4.5 PFLOP/s (no measured fp8 peak)"))
    traffic = load_traffic()
    entry = ((traffic or {}).get("ops") or {}).get(name) if not fp8 else None
    tr = entry.get("bytes_per_launch") if entry else None
    return {"bound": "tensor", "kernel": name, "achieved": ach, "peak": peak, "unit": "TFLOP/s",
            "frac": ach / peak, "peak_source": peak_name,
            "frac_of_sustained": ach / peaks["bf16_tflops_sustained"],
            "traffic": tr,
            "traffic_source": (f"{traffic['what']}; this launch: {entry['captured_read_bytes'] / 1e6:.0f} MB read + "
                               f"{entry['captured_write_bytes'] / 1e6:.0f} MB written = {entry['ratio_to_algorithmic']}x "
                               f"its algorithmic bytes {entry['algorithmic_formula']}") if tr else None,
            "algorithmic_flop_per_launch": fl,
            "ops": {k: {"avg_ms": round(v["avg_ms"], 4), "launches": v["launches"],
                        "ms_per_step": round(per_step_ms(v), 4),
                        "tflops": OP_FLOP_UNITS.get(k, 0) * float(local_rows) * H * I / (per_step_ms(v) * 1e-3) / 1e12}
                    for k, v in ops.items()}}


def single_gpu_setup(args, wl, E, zero, tokens, topk, H, I, zipf_s, device):
    """Seeded routing, inputs and weights of a 1-GPU workload on `device`."""
    import torch

    from cutlass_op.bf16_grouped_mm.workloads import (MoEShape, config5_counts, make_weights_device,
                                                      offs_from_counts, zipf_routing)

    if wl == "cfg5":
        counts = config5_counts(tokens, E, topk, seed=0)
    else:
        counts = zipf_routing(tokens, E, topk, zipf_s, seed=0, zero_experts=zero)
    M = int(counts.sum())
    offs = offs_from_counts(counts).to(device)
    gx = torch.Generator(device=device).manual_seed(1)
    x = torch.randn(M, H, generator=gx, device=device).to(torch.bfloat16).requires_grad_(True)
    w_up, b_up, w_down, b_down = [t.requires_grad_(True) for t in
                                  make_weights_device(MoEShape(E, H, I), seed=2, device=device)]
    return counts, M, offs, x, w_up, b_up, w_down, b_down


def ffn_step_fn(mgf, params, offs, fwd_only=False, recompute=False):
    import torch

    x, w_up, b_up, w_down, b_down = params

    def step():
        for p in params:
            p.grad = None
        if fwd_only:
            with torch.no_grad():
                mgf.grouped_mm_swiglu(x, w_up, offs, b_up, ALPHA, LIMIT)
            return
        if recompute:
            out = mgf.grouped_mm_ffn(x, w_up, w_down, offs, b_up, b_down, ALPHA, LIMIT, store_aux=False)
        else:
            s_, aux = mgf.grouped_mm_swiglu(x, w_up, offs, b_up, ALPHA, LIMIT)
            out = mgf.grouped_mm_downproj(s_, w_down, offs, b_down, aux, ALPHA, LIMIT)
        out.sum().backward()
    return step


def extra_workloads(args, mgf, device, peaks, peak_src):
    """Secondary 1-GPU measurements carried in the same JSON line (not the headline): config 2
    (forward only), config 5 at 4096 tokens (the HBM-bound fine-grained corner) and config 4's
    one-GPU point (E=128 through the expert-parallel module on one rank: the N=1 anchor of the
    expert-parallel scaling curve)."""
    import torch

    from cutlass_op.bf16_grouped_mm.optimer import OpTimer

    steps, warm = max(3, min(args.steps, 20)), max(3, min(args.warmup, 5))
    out = {}
    for name, wl, E, zero, tokens, topk, H, I, zs, fwd in (
            ("cfg2_fwd", "cfg2", 32, 0, 24576, 4, 2880, 2880, 1.1, True),
            ("cfg5_t4096", "cfg5", 256, 0, 4096, 8, 7168, 2048, 1.3, False)):
        try:
            counts, M, offs, x, w_up, b_up, w_down, b_down = single_gpu_setup(
                args, wl, E, zero, tokens, topk, H, I, zs, device)
            step = ffn_step_fn(mgf, [x, w_up, b_up, w_down, b_down], offs, fwd_only=fwd)
            for _ in range(warm):
                step()
            timer = OpTimer().install()
            ms = time_steps(step, steps, 0)
            timer.uninstall()
            fl = (4.0 if fwd else 18.0) * M * H * I
            roof = roofline_entry(timer.summary(), M, H, I, peaks, peak_src, steps=steps)
            out[name] = {"ms_per_step": ms, "tflops": fl / (ms * 1e-3) / 1e12, "routed_rows": M, "steps": steps,
                         "E": E, "H": H, "I": I, "tokens": tokens, "topk": topk,
                         "ops": roof["ops"] if roof else None}
            del x, w_up, b_up, w_down, b_down, step
        except Exception as e:  # report, do not fail the bench
            out[name] = {"error": f"{type(e).__name__}: {str(e)[:200]}"}
        torch.cuda.empty_cache()
    # the cfg3 FFN with every forward and backward GEMM in e4m3 (quantisation inside the step), next to
    # a measured cuBLAS e4m3 GEMM peak (torch._scaled_mm, 8192^3, best of 10) as its denominator
    try:
        from cutlass_op.bf16_grouped_mm import fp8 as fp8_mod

        counts, M, offs, x, w_up, b_up, w_down, b_down = single_gpu_setup(
            args, "cfg3", 32, 2, 24576, 4, 2880, 2880, 1.1, device)
        params = [x, w_up, b_up, w_down, b_down]

        def step():
            for p_ in params:
                p_.grad = None
            fp8_mod.grouped_mm_ffn_fp8(x, w_up, w_down, offs, b_up, b_down, ALPHA, LIMIT).sum().backward()
        for _ in range(warm):
            step()
        timer = OpTimer().install()
        ms = time_steps(step, steps, 0)
        timer.uninstall()
        fp8_ops = {k: round(v["avg_ms"], 4) for k, v in timer.summary().items()}
        fp8_launches = {k: v["launches"] // steps for k, v in timer.summary().items()}
        del x, w_up, b_up, w_down, b_down, params, step
        torch.cuda.empty_cache()
        peak8 = measure_e4m3_peak(device)
        tf = 18.0 * M * 2880 * 2880 / (ms * 1e-3) / 1e12
        out["cfg3_fp8_ffn"] = {"ms_per_step": ms, "tflops": tf, "measured_e4m3_peak_tflops": peak8,
                               "ops_avg_ms": fp8_ops, "ops_per_step": fp8_launches,
                               "frac_of_measured_e4m3_peak": tf / peak8,
                               "what": "grouped_mm_ffn_fp8 fwd+bwd at cfg3 (every GEMM e4m3, bf16 in/out, "
                                       "quantisers inside the step); peak = torch._scaled_mm e4m3 8192^3 burst"}
    except Exception as e:
        out["cfg3_fp8_ffn"] = {"error": f"{type(e).__name__}: {str(e)[:200]}"}
    torch.cuda.empty_cache()
    try:
        from cutlass_op.bf16_grouped_mm.expert_parallel import EPMoEFFN, route_tokens

        E, H, I, T, K = 128, 2880, 2880, 24576, 4
        res = {}
        for routing in ("uniform", "zipf"):
            ffn = EPMoEFFN(E, H, I, group=None, device=device, seed=2)
            x = torch.randn(T, H, generator=torch.Generator(device=device).manual_seed(1), device=device)
            x = x.to(torch.bfloat16).requires_grad_(True)
            idx = route_tokens(T, E, K, routing, seed=100, device=device)

            def step():
                x.grad = None
                ffn.zero_grad()
                ffn(x, idx).sum().backward()
            for _ in range(warm):
                step()
            ms = time_steps(step, steps, 0)
            res[routing] = {"ms_per_step": ms, "tflops": 18.0 * T * K * H * I / (ms * 1e-3) / 1e12}
            del ffn, x, step
            torch.cuda.empty_cache()
        out["cfg4_n1"] = dict(res, what="cfg4 at N=1: E=128 H=I=2880, 24576 tokens top-4 through EPMoEFFN on "
                                        "one rank (local gather/permute/combine, no exchange)")
    except Exception as e:
        out["cfg4_n1"] = {"error": f"{type(e).__name__}: {str(e)[:200]}"}
    return out


def main():
    args = parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.cpu_baseline_only:
        print(json.dumps(cpu_sample_tflops(args, 1)), flush=True)
        return
    if args.impl == "reference":
        if rank != 0:
            return
        _reexec_with_malloc_env()
        reference_arm(args, rank, world)
        return

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=device)
    barrier = (lambda: dist.barrier()) if world > 1 else None

    import cutlass_op.bf16_grouped_mm as mgf
    from cutlass_op.bf16_grouped_mm.optimer import OpTimer

    wl, desc, E_total, zero, tokens, topk, H, I, zipf_s, fwd_only = build_workload(args, rank, world, device)
    peaks, peak_src = load_peaks()
    ep_parity = None

    if world == 1:
        E = E_total
        counts, M, offs, x, w_up, b_up, w_down, b_down = single_gpu_setup(
            args, wl, E, zero, tokens, topk, H, I, zipf_s, device)
        params = [x, w_up, b_up, w_down, b_down]
        if args.fp8:
            if not fwd_only:
                raise SystemExit("--fp8 needs --workload cfg2 (the FP8 operators are forward-only)")
            from cutlass_op.bf16_grouped_mm import fp8 as fp8_mod

            with torch.no_grad():
                qx, sx = fp8_mod.quantize_rows(x.detach())
                qw, sw = fp8_mod.quantize_weights(w_up.detach())

            def step():
                with torch.no_grad():
                    fp8_mod.grouped_mm_swiglu_fp8(qx, qw, offs, sx, sw, b_up, ALPHA, LIMIT)
        else:
            step = ffn_step_fn(mgf, params, offs, fwd_only=fwd_only, recompute=args.recompute_aux)
        local_rows = M
    else:
        from cutlass_op.bf16_grouped_mm.expert_parallel import EPMoEFFN, route_tokens

        ep_parity = ep_parity_check(args, world, rank, device)
        torch.cuda.empty_cache()
        ffn = EPMoEFFN(E_total, H, I, group=None, device=device, seed=2, transport=args.transport,
                       overlap=args.ep_overlap, fused=not args.ep_unfused, pipeline=args.ep_pipeline)
        gx = torch.Generator(device=device).manual_seed(1 + rank)
        x = torch.randn(tokens, H, generator=gx, device=device).to(torch.bfloat16).requires_grad_(True)
        expert_idx = route_tokens(tokens, E_total, topk, args.routing, seed=100 + rank, device=device)

        def step():
            x.grad = None
            ffn.zero_grad()
            out = ffn(x, expert_idx)
            out.sum().backward()
        local_rows = None

    # warm-up + timed region (device-resident inputs, larger than L2)
    timer = OpTimer()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    clocks = None
    sampler = None
    if rank == 0:
        uuid = str(torch.cuda.get_device_properties(device).uuid)
        sampler = ClockSampler(uuid if uuid.startswith("GPU-") else f"GPU-{uuid}")
        sampler.start()
    timer.install()
    ms = time_steps(step, args.steps, 0, barrier)
    timer.uninstall()
    if sampler is not None:
        clocks = sampler.stop()
    ops = timer.summary()
    if world > 1:
        local_rows = int(ffn.last_local_rows)
    flops_local = (4.0 if fwd_only else 18.0) * local_rows * H * I
    t = torch.tensor([ms, flops_local], dtype=torch.float64, device=device)
    if world > 1:
        tmax = t.clone()
        dist.all_reduce(tmax[:1], op=dist.ReduceOp.MAX)
        tsum = t.clone()
        dist.all_reduce(tsum[1:], op=dist.ReduceOp.SUM)
        ms_max, flops_all = float(tmax[0]), float(tsum[1])
    else:
        ms_max, flops_all = ms, flops_local
    value = flops_all / (ms_max * 1e-3) / 1e12
    per_gpu = value / world
    ours_launches = sum(v["launches"] for k, v in ops.items() if k in OP_FLOP_UNITS or k.startswith("ep_"))
    peak8 = measure_e4m3_peak(device) if args.fp8 and ops else None
    roof = (roofline_entry(ops, local_rows, H, I, peaks, peak_src, fp8=args.fp8, steps=args.steps, fp8_peak=peak8)
            if ops else None)

    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "e4m3 x e4m3 -> fp32 accumulate, bf16 out" if args.fp8 else "bf16",
        "data": "synthetic (seeded, shapes of the configured workload)",
        "config": line_config(args, world),
        "routed_rows_gpu0": local_rows,
        "tflops_per_gpu": per_gpu,
        "pct_of_peak": 100.0 * per_gpu / (peak8 if peak8 else peaks["bf16_tflops"]),
        "peak_tflops": peak8 if peak8 else peaks["bf16_tflops"],
        "peak_source": ("measured e4m3 burst (torch._scaled_mm 8192^3 on this GPU)" if peak8 else
                        f"{peak_src} bf16_tflops (burst)"),
        "pct_of_sustained_peak": 100.0 * per_gpu / peaks["bf16_tflops_sustained"],
        "gpu_launches": int(ours_launches),
        "roofline": roof,
        "clocks": clocks,
    }
    if ep_parity is not None:
        line["ep_parity"] = ep_parity
    if world > 1 and ops:
        # step time split by kind, rank 0's view: grouped GEMMs vs expert-parallel plan / row movement /
        # waits; the GEMM time scaled to the max SM clock separates clock from communication effects
        gemm = sum(v["total_ms"] for k, v in ops.items() if k in OP_FLOP_UNITS) / args.steps
        comm = sum(v["total_ms"] for k, v in ops.items() if k.startswith("ep_")) / args.steps
        mhz = (clocks or {}).get("sm_mhz")
        line["ep_breakdown"] = {
            "gemm_ms_per_step": gemm, "ep_ms_per_step": comm, "other_ms_per_step": ms - gemm - comm,
            "sm_mhz_median": mhz,
            "gemm_ms_at_max_clock": gemm * mhz / 1965.0 if mhz else None,
            "ep_ops_ms_per_step": {k: round(v["total_ms"] / args.steps, 4) for k, v in ops.items() if k.startswith("ep_")}}

    # torch._grouped_mm + eager bias/SwiGLU on the same inputs (single GPU only)
    if world == 1 and not args.no_compare and not args.fp8:
        line["torch_grouped_mm"] = compare_torch(step_inputs=(x, w_up, b_up, w_down, b_down, offs, counts),
                                                 steps=args.steps, warmup=args.warmup, flops=flops_local,
                                                 fwd_only=fwd_only)

    # end-to-end through the public API with host buffers
    if world == 1 and not args.no_e2e and not args.fp8:
        line["e2e"] = e2e_run(mgf, x, w_up, b_up, w_down, b_down, offs, counts, args, flops_local, fwd_only)
    elif world > 1 and not args.no_e2e:
        e2e = e2e_run_ep(ffn, x, expert_idx, args, barrier)
        t = torch.tensor([e2e["ms_per_step"]], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e["ms_per_step"] = float(t[0])
        e2e["value"] = flops_all / (e2e["ms_per_step"] * 1e-3) / 1e12
        e2e["unit"] = UNIT
        if rank == 0:
            line["e2e"] = e2e

    if world == 1 and not args.no_extra and wl == "cfg3" and not args.tokens and not args.experts:
        del step
        params = x = w_up = b_up = w_down = b_down = None
        torch.cuda.empty_cache()
        line["extra"] = extra_workloads(args, mgf, device, peaks, peak_src)

    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_subprocess(args)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def compare_torch(step_inputs, steps, warmup, flops, fwd_only=False):
    """torch._grouped_mm + eager bias / clamped SwiGLU / autograd on the same inputs and GPU.

    Three forms of the same step are timed:
      * ``ms_per_step`` (the comparator): per-row biases gathered as b[row_expert] and added
        (one [M, N] gather per bias; the fastest eager form measured here);
      * ``inplace_bias_ms``: the biases added in place, one row block per expert (no gathered
        tensor, but E small kernels and their autograd copies);
      * ``grouped_mm_only_ms``: the graph without bias and SwiGLU -- the two torch._grouped_mm GEMMs
        and their autograd alone (same FLOPs), so ``eager_ops_ms`` = comparator - this is the time
        of the unfused eager operations."""
    import torch

    x, w_up, b_up, w_down, b_down, offs, counts = step_inputs
    try:
        bounds = torch.cumsum(counts.cpu(), 0).tolist()
        starts = [0] + bounds[:-1]
        row_e = torch.repeat_interleave(torch.arange(len(counts), device=x.device), counts.to(x.device))
        xs = x.detach().clone().requires_grad_(True)
        wu, bu, wd, bd = [t.detach().clone().requires_grad_(True) for t in (w_up, b_up, w_down, b_down)]
        params = [xs, wu, bu, wd, bd]
        ones = torch.ones(x.shape[0], w_down.shape[-1], dtype=x.dtype, device=x.device)

        def add_bias(h, b, mode):
            if mode == "gather":
                return h + b[row_e]
            for e, (s0, s1) in enumerate(zip(starts, bounds)):  # in place on each expert's row block
                if s1 > s0:
                    h[s0:s1] += b[e]
            return h

        def make(mode):
            def step():
                for p in params:
                    p.grad = None
                ctx = torch.no_grad() if fwd_only else torch.enable_grad()
                with ctx:
                    h = torch._grouped_mm(xs, wu, offs=offs)
                    if mode != "gemm_only":
                        h = add_bias(h, bu, mode)
                        g = h[:, 0::2].clamp(max=LIMIT)
                        u = h[:, 1::2].clamp(min=-LIMIT, max=LIMIT)
                        s_ = g * torch.sigmoid(ALPHA * g) * (u + 1.0)
                    else:
                        s_ = h[:, 0::2].contiguous()
                    if fwd_only:
                        return
                    out = torch._grouped_mm(s_, wd, offs=offs)
                    if mode != "gemm_only":
                        out = add_bias(out, bd, mode)
                    # d(out.sum())/d(out) as a materialised tensor: torch._grouped_mm's backward rejects the
                    # zero-stride expanded gradient that out.sum().backward() produces.
                    out.backward(ones)
            return step

        ms = time_steps(make("gather"), steps, warmup)
        short = max(3, steps // 3)
        ms_inplace = time_steps(make("inplace"), short, min(warmup, 3))
        ms_gemm = time_steps(make("gemm_only"), short, min(warmup, 3))
        return {"ms_per_step": ms, "value": flops / (ms * 1e-3) / 1e12, "unit": UNIT,
                "inplace_bias_ms": ms_inplace, "grouped_mm_only_ms": ms_gemm, "eager_ops_ms": ms - ms_gemm,
                "what": "torch._grouped_mm + eager gathered per-row bias / clamped SwiGLU / autograd, same inputs, "
                        "same GPU; inplace_bias_ms = biases added in place per expert block; grouped_mm_only_ms = the "
                        "two grouped GEMMs and their autograd without bias and SwiGLU; eager_ops_ms = the difference"}
    except Exception as e:  # report, do not fail the bench
        return {"error": f"{type(e).__name__}: {str(e)[:200]}"}


def e2e_run(mgf, x, w_up, b_up, w_down, b_down, offs, counts, args, flops, fwd_only=False):
    """Public-API step with the step's inputs copied from pinned host memory and the loss read back.

    Every step copies its x rows and offs host -> device and reads the loss device -> host.  The
    copies run on a copy stream into the other of two device buffers while the previous step
    computes (a data prefetcher), and the timed window ends only after the last of them has landed:
    K timed steps hold K full host -> device copies and K fwd+bwd passes.
    """
    import torch

    x_host = x.detach().to("cpu").pin_memory()
    offs_host = offs.to("cpu").pin_memory()
    loss_host = torch.empty((), dtype=torch.float32).pin_memory()
    x_dev = [torch.empty_like(x.detach()) for _ in range(2)]
    offs_dev = [torch.empty_like(offs) for _ in range(2)]
    ready = [torch.cuda.Event() for _ in range(2)]
    free = [torch.cuda.Event() for _ in range(2)]
    copy_stream = torch.cuda.Stream()
    params = [w_up, b_up, w_down, b_down]
    state = {"i": 0}

    def issue_copy(slot):
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(free[slot])  # the step that last read this buffer is done
            x_dev[slot].copy_(x_host, non_blocking=True)
            offs_dev[slot].copy_(offs_host, non_blocking=True)
            ready[slot].record(copy_stream)

    issue_copy(0)

    def step():
        slot = state["i"] & 1
        state["i"] += 1
        issue_copy(slot ^ 1)  # the next step's inputs, under this step's compute
        torch.cuda.current_stream().wait_event(ready[slot])
        for p in params:
            p.grad = None
        xs, os_ = x_dev[slot], offs_dev[slot]
        if fwd_only:
            with torch.no_grad():
                s, _ = mgf.grouped_mm_swiglu(xs, w_up, os_, b_up, ALPHA, LIMIT)
                loss_host.copy_(s.sum(dtype=torch.float32), non_blocking=True)
        else:
            xl = xs.detach().requires_grad_(True)
            s, aux = mgf.grouped_mm_swiglu(xl, w_up, os_, b_up, ALPHA, LIMIT)
            out = mgf.grouped_mm_downproj(s, w_down, os_, b_down, aux, ALPHA, LIMIT)
            loss = out.sum(dtype=torch.float32)
            loss.backward()
            loss_host.copy_(loss.detach(), non_blocking=True)
        free[slot].record()

    def tail():
        torch.cuda.current_stream().wait_stream(copy_stream)

    ms = time_steps(step, args.steps, args.warmup, tail=tail)
    return {"value": flops / (ms * 1e-3) / 1e12, "unit": UNIT, "ms_per_step": ms,
            "h2d_bytes_per_step": x_host.numel() * x_host.element_size() + offs_host.numel() * 4,
            "d2h_bytes_per_step": 4,
            "h2d": "pinned host -> device on a copy stream, one step ahead (double-buffered prefetch)"}


def e2e_run_ep(ffn, x, expert_idx, args, barrier):
    """Expert-parallel step through EPMoEFFN with each rank's token rows and routing copied from pinned
    host memory every step (on a copy stream, one step ahead, double-buffered, the last copy inside
    the timed window) and the loss read back.  Returns this rank's ms per step; the caller takes the
    max over ranks."""
    import torch

    x_host = x.detach().to("cpu").pin_memory()
    idx_host = expert_idx.to("cpu").pin_memory()
    loss_host = torch.empty((), dtype=torch.float32).pin_memory()
    x_dev = [torch.empty_like(x.detach()) for _ in range(2)]
    idx_dev = [torch.empty_like(expert_idx) for _ in range(2)]
    ready = [torch.cuda.Event() for _ in range(2)]
    free = [torch.cuda.Event() for _ in range(2)]
    copy_stream = torch.cuda.Stream()
    state = {"i": 0}

    def issue_copy(slot):
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(free[slot])
            x_dev[slot].copy_(x_host, non_blocking=True)
            idx_dev[slot].copy_(idx_host, non_blocking=True)
            ready[slot].record(copy_stream)

    issue_copy(0)

    def step():
        slot = state["i"] & 1
        state["i"] += 1
        issue_copy(slot ^ 1)
        torch.cuda.current_stream().wait_event(ready[slot])
        ffn.zero_grad()
        xl = x_dev[slot].detach().requires_grad_(True)
        loss = ffn(xl, idx_dev[slot]).sum(dtype=torch.float32)
        loss.backward()
        loss_host.copy_(loss.detach(), non_blocking=True)
        free[slot].record()

    def tail():
        torch.cuda.current_stream().wait_stream(copy_stream)

    ms = time_steps(step, args.steps, args.warmup, barrier=barrier, tail=tail)
    return {"ms_per_step": ms,
            "h2d_bytes_per_step": x_host.numel() * x_host.element_size() + idx_host.numel() * idx_host.element_size(),
            "d2h_bytes_per_step": 4,
            "h2d": "per rank: pinned host -> device on a copy stream, one step ahead (double-buffered prefetch)"}


if __name__ == "__main__":
    main()
