"""Stages lightserve's own Triton kernels, unmodified, for the same-box
comparison test (tests/test_gpu_reference_triton.py) and bench.py's
`reference_triton` context line.

lightserve has neither setup.py nor pyproject.toml, so it cannot be
pip-installed; this copies the three kernel modules of the attention path
verbatim into baseline/_ref/kernels/ (git-ignored, never committed, carried to
the GPU box with the working tree) with an empty __init__.py so that
`import kernels.flash_attention` works from baseline/_ref. Nothing in the
lightserve_b200 package imports them.

    python tests/stage_reference_kernels.py --reference <lightserve checkout>
"""
from __future__ import annotations

import argparse
import shutil
from pathlib import Path

FILES = ("flash_attention.py", "flash_attention_backward.py", "fused_rmsnorm_residual.py")
DEST = Path(__file__).resolve().parent.parent / "baseline" / "_ref" / "kernels"


def main():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", required=True, help="path of the lightserve source tree")
    args = ap.parse_args()
    src = Path(args.reference) / "kernels"
    DEST.mkdir(parents=True, exist_ok=True)
    for f in FILES:
        shutil.copyfile(src / f, DEST / f)
    (DEST / "__init__.py").write_text("")
    print(f"staged {', '.join(FILES)} -> {DEST}")


if __name__ == "__main__":
    main()
