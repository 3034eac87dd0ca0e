"""Failure detection on the GPU without a fault: a kernel whose pipeline waits run out.

With MGF_TEST_STALL_PRODUCER=1 the producer warp hands out no tiles, so the MMA and epilogue warps'
bounded waits give up after their 1.5 s limit.  The kernel must then record MGF_DEV_WAIT_TIMEOUT,
free its tensor memory and return; the CUDA context stays usable, shown by a correct GEMM launched
in the same process afterwards.  Runs in a child process so the environment switch stays local.
"""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

REPO = Path(__file__).resolve().parent.parent

CHILD = r'''
import json, os, sys, time
sys.path[:0] = [sys.argv[1], os.path.join(sys.argv[1], "cute-moe-train_b200")]
import torch
import cutlass_op.bf16_grouped_mm as m
from cutlass_op.bf16_grouped_mm.workloads import small_case
from oracle import moe_ffn as O
x, w, b, _, _, offs, _ = small_case(2, 128, 64, [100, 60], seed=1)
xd, wd, bd, od = x.cuda(), w.cuda(), b.cuda(), offs.cuda()
m.device_status()  # clear
os.environ["MGF_TEST_STALL_PRODUCER"] = "1"
t0 = time.time()
m.grouped_mm(xd, wd, od, bd)
torch.cuda.synchronize()
stalled_s = time.time() - t0
status = m.device_status()
os.environ["MGF_TEST_STALL_PRODUCER"] = "0"
out = m.grouped_mm(xd, wd, od, bd)
torch.cuda.synchronize()
after = m.device_status()
r = O.check("after", out.float().cpu(), O.grouped_linear(x, w, offs, b))
print(json.dumps({"stalled_s": stalled_s, "status": status, "after_status": after, "ok": r["ok"], "rel": r["rel"]}))
'''


def test_bounded_waits_report_and_recover():
    env = dict(os.environ)
    res = subprocess.run([sys.executable, "-c", CHILD, str(REPO)], env=env, capture_output=True, text=True, timeout=120)
    assert res.returncode == 0, res.stderr[-2000:]
    d = json.loads(res.stdout.strip().splitlines()[-1])
    assert d["status"] & 0x1, d              # MGF_DEV_WAIT_TIMEOUT recorded
    assert 1.0 < d["stalled_s"] < 30.0, d    # gave up after its limit instead of hanging
    assert d["after_status"] == 0 and d["ok"], d
