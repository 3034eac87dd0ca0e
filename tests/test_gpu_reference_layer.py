"""The reference's own Python layer driving this repository's kernels through the C ABI.

The reference package's unmodified __init__.py + custom_op.py (the staged copy under
baseline/_ref/group_gemm, written by baseline/stage_reference.py) are imported with
cute-moe-train_b200/ctypes_ext.py as their `_ext` -- the binding a maintainer would drop into the
reference.  Config 1 (E=8, H=2048, I=1024, the reference quick-start token counts incl. an empty
expert) then runs forward and backward through the reference's autograd graph on the GPU and every
output and gradient is checked against the oracle (max|err|/max|ref| <= 1e-2, cosine >= 0.9999).
It runs in a child process that never loads this repository's torch operators, because the
reference layer registers the same `grouped_mm` namespace.
"""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
STAGED = REPO / "baseline" / "_ref" / "group_gemm"

CHILD = r"""
import json, sys
from pathlib import Path
repo = Path(sys.argv[1])
sys.path[:0] = [str(repo), str(repo / "cute-moe-train_b200")]
import importlib.util, torch
spec = importlib.util.spec_from_file_location("ref_pkg._ext", repo / "cute-moe-train_b200" / "ctypes_ext.py")
ext = importlib.util.module_from_spec(spec); spec.loader.exec_module(ext)
from oracle.ref_ext_cpu import load_reference_layer
from oracle import moe_ffn as O
ref = load_reference_layer(repo / "baseline" / "_ref" / "group_gemm", ext=ext, modname="ref_pkg")
assert "cutlass_op" not in sys.modules
spec = importlib.util.spec_from_file_location("wl", repo / "cute-moe-train_b200" / "cutlass_op" / "bf16_grouped_mm" / "workloads.py")
wl = importlib.util.module_from_spec(spec); sys.modules["wl"] = wl; spec.loader.exec_module(wl)
x, w_up, b_up, w_down, b_down, offs = wl.config1()
gout = torch.randn(x.shape[0], x.shape[1], generator=torch.Generator().manual_seed(7)).to(torch.bfloat16)
dev = torch.device("cuda", 0)
leaves = [t.to(dev).requires_grad_(True) for t in (x, w_up, b_up, w_down, b_down)]
xl, wu, bu, wd, bd = leaves
od = offs.to(dev)
s, aux = ref.grouped_mm_swiglu(xl, wu, offs=od, bias=bu, swiglu_alpha=1.702, swiglu_limit=7.0)
out = ref.grouped_mm_downproj(s, wd, offs=od, bias=bd, aux_biased_acc=aux, swiglu_alpha=1.702, swiglu_limit=7.0)
out.backward(gout.to(dev))
torch.cuda.synchronize()
want = O.kernel_chain(x, w_up, b_up, w_down, b_down, offs, gout)
got = {"swiglu_out": s, "aux": aux, "out": out, "dx": xl.grad, "dw_up": wu.grad, "db_up": bu.grad,
       "dw_down": wd.grad, "db_down": bd.grad}
res = {k: O.check(k, v.detach().float().cpu(), want[k]) for k, v in got.items()}
empty = [e for e, n in enumerate(wl.CONFIG1_TPE) if n == 0]
res["empty_expert_zero"] = {"ok": all(int(torch.count_nonzero(got[k][e])) == 0 for e in empty
                                      for k in ("dw_up", "db_up", "dw_down", "db_down"))}
res["ops_loaded"] = {"ok": not any("_grouped_mm_ops" in str(getattr(m, "__file__", "")) for m in sys.modules.values())}
print("RESULT " + json.dumps(res))
"""


@pytest.mark.gpu
@pytest.mark.skipif(not (STAGED / "custom_op.py").is_file(), reason="reference layer not staged (baseline/_ref)")
def test_reference_python_layer_over_ctypes_binding():
    r = subprocess.run([sys.executable, "-c", CHILD, str(REPO)], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    line = next(ln for ln in r.stdout.splitlines() if ln.startswith("RESULT "))
    res = json.loads(line[len("RESULT "):])
    bad = {k: v for k, v in res.items() if not v["ok"]}
    assert not bad, bad
