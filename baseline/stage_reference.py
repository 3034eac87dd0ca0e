"""Stage the reference implementation under baseline/_ref (git-ignored; it travels with the tree).

    python baseline/stage_reference.py [REF_ROOT]

1. Runs the reference's own install, ``pip install --no-index --no-build-isolation --find-links
   /opt/wheelhouse --target baseline/_ref <REF_ROOT>/cutlass_op/bf16_grouped_mm``.  Its setup.py
   builds an sm_90a CUDA extension from a CUTLASS fork that the checkout does not vendor, so the
   install stops at "CUTLASS headers not found"; the outcome is recorded in baseline/_ref/STAGED.json.
2. When it fails, places the package's pure-Python layer -- ``__init__.py`` and ``custom_op.py``,
   byte for byte -- in baseline/_ref/group_gemm/ (the package name its setup.py installs), with their
   sha256 in STAGED.json.  That is the part of the install that needs no compiler.

bench.py's reference arm and tests/test_gpu_reference_layer.py import that layer from there, with
``_ext`` supplied from this repository (a CPU restatement of the three kernels, or the ctypes
binding of libmoe_gemm.so).  Nothing at run time reads REF_ROOT.
"""

from __future__ import annotations

import hashlib
import json
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REF_DIR = HERE / "_ref"
PKG_DIR = REF_DIR / "group_gemm"
STAMP = REF_DIR / "STAGED.json"
FILES = ("__init__.py", "custom_op.py")
DEFAULT_REF_ROOT = Path(os.environ.get("MGF_REFERENCE_ROOT", "/root/reference"))


def _sha(p: Path) -> str:
    return hashlib.sha256(p.read_bytes()).hexdigest()


def staged() -> dict | None:
    """The STAGED.json record when the staged layer is present and unaltered, else None."""
    if not STAMP.is_file():
        return None
    rec = json.loads(STAMP.read_text())
    for f in FILES:
        p = PKG_DIR / f
        if not p.is_file() or _sha(p) != rec.get("sha256", {}).get(f):
            return None
    return rec


def stage(ref_root: Path = DEFAULT_REF_ROOT, verbose: bool = True) -> dict | None:
    src = ref_root / "cutlass_op" / "bf16_grouped_mm"
    if not src.is_dir():
        return staged()
    rec = staged()
    if rec is not None and all(rec["sha256"][f] == _sha(src / f) for f in FILES):
        return rec
    REF_DIR.mkdir(parents=True, exist_ok=True)
    cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--find-links",
           "/opt/wheelhouse", "--target", str(REF_DIR), str(src)]
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
        rc, out = r.returncode, (r.stdout + r.stderr)
    except Exception as e:  # pip missing, timeout
        rc, out = -1, f"{type(e).__name__}: {e}"
    why = next((ln.strip() for ln in out.splitlines() if "CUTLASS headers not found" in ln), None)
    if why is None:
        why = next((ln.strip() for ln in reversed(out.splitlines()) if "error" in ln.lower()), out[-300:])
    PKG_DIR.mkdir(parents=True, exist_ok=True)
    for f in FILES:
        shutil.copyfile(src / f, PKG_DIR / f)
    rec = {"pip_install_rc": rc, "pip_install_outcome": "ok" if rc == 0 else f"failed: {why}",
           "staged": "pure-Python layer copied byte for byte (the compiled _ext cannot be built)",
           "files": list(FILES), "sha256": {f: _sha(PKG_DIR / f) for f in FILES}}
    STAMP.write_text(json.dumps(rec, indent=1))
    if verbose:
        print(f"baseline/_ref: pip install rc={rc}; staged {', '.join(FILES)} into {PKG_DIR}")
    return rec


if __name__ == "__main__":
    print(json.dumps(stage(Path(sys.argv[1]) if len(sys.argv) > 1 else DEFAULT_REF_ROOT), indent=1))
