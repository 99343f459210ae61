"""Stage the reference's own CPU implementation of this path into ``oracle/_ref``.

TEST INFRASTRUCTURE ONLY (the timed CPU baseline of ``bench.py`` and the
reference arm ``bench.py --impl reference``).  The reference path is Python
(``cutechronos.model.CuteChronos2Model`` with its torch fallbacks on CPU
tensors), so "building" it means copying the package's Python sources, as they
lie in the reference checkout, into the git-ignored ``oracle/_ref/`` folder;
that folder travels with the working tree to a GPU box, where the checkout
itself does not exist.  Nothing of it is committed and the product never
imports it.

Usage:  python oracle/stage_reference.py [--reference <checkout>]
"""

from __future__ import annotations

import argparse
import shutil
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
DEFAULT_REF = Path("/root/reference")
# the sub-packages ``cutechronos.model`` imports (its kernel dispatch imports
# the Triton / CuTe modules at import time; on CPU tensors it runs the torch
# fallbacks)
PARTS = ("__init__.py", "model.py", "kernel_backends.py", "kernels.py", "pipeline.py",
         "modules", "triton_kernels", "cutlass_kernels")


def stage(reference: Path = DEFAULT_REF) -> Path | None:
    src = reference / "cutechronos"
    if not (src / "model.py").exists():
        return None
    dst = OUT / "cutechronos"
    if dst.exists():
        shutil.rmtree(dst)
    dst.mkdir(parents=True)
    for part in PARTS:
        p = src / part
        if p.is_dir():
            shutil.copytree(p, dst / part, ignore=shutil.ignore_patterns("__pycache__", "tests", "*.so"))
        elif p.exists():
            shutil.copy2(p, dst / part)
    (OUT / "SOURCE.txt").write_text(f"staged from {src} by oracle/stage_reference.py\n")
    return dst


def load_reference_model_class():
    """CuteChronos2Model / CuteChronos2Config of the staged reference, or None."""
    if not (OUT / "cutechronos" / "model.py").exists():
        return None
    if str(OUT) not in sys.path:
        sys.path.insert(0, str(OUT))
    from cutechronos.model import CuteChronos2Config, CuteChronos2Model  # noqa: E402
    return CuteChronos2Config, CuteChronos2Model


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, default=DEFAULT_REF)
    a = ap.parse_args()
    print(stage(a.reference) or "reference checkout not found; nothing staged")
