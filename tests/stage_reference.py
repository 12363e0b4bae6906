"""Stage an unmodified copy of the reference project next to this repository.

    python tests/stage_reference.py --reference PATH_TO_REFERENCE_CHECKOUT

Installs the reference (sahan974/DeepSeek-V2-Lite-CUDA: its pure-PyTorch modules
`reference.{moe,mla,decoder_layer}` and `kernels.*`) into baseline/_ref with pip, and puts its
own test scripts, unmodified, in baseline/_ref/tests/.  baseline/_ref is git-ignored, so
nothing of the reference enters this repository's history, but it travels with the working
tree to a GPU machine, where

  * tests/test_reference_scripts_gpu.py runs each of the reference's kernel test scripts as a
    subprocess against this package's `ds_kernels` / `moe_fused` (the drop-in check), and
  * `bench.py --impl reference` and the benchmark's `cpu_baseline` time the reference's own
    CPU module `DeepSeekMoE` (src/reference/moe.py) on the benchmark workload.

The install is the plain pip form: no index, no build isolation, no dependencies (torch and
numpy are already present); the checkout is copied to a temporary directory first because
the build writes into its source tree.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import tempfile

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DEST = os.path.join(ROOT, "baseline", "_ref")


def stage(reference: str, dest: str = DEST) -> str:
    if not os.path.isfile(os.path.join(reference, "src", "reference", "moe.py")):
        raise SystemExit(f"{reference} does not look like the reference checkout "
                         "(src/reference/moe.py missing)")
    with tempfile.TemporaryDirectory() as tmp:
        src = os.path.join(tmp, "reference")
        shutil.copytree(reference, src, ignore=shutil.ignore_patterns(".git", "build"))
        for d, _, files in os.walk(src):
            os.chmod(d, 0o755)
            for f in files:
                os.chmod(os.path.join(d, f), 0o644)
        if os.path.isdir(dest):
            shutil.rmtree(dest)
        subprocess.run([sys.executable, "-m", "pip", "install", "--no-index",
                        "--no-build-isolation", "--no-deps", "--quiet", "--target", dest, src],
                       check=True)
    tests = os.path.join(dest, "tests")
    os.makedirs(tests, exist_ok=True)
    for f in sorted(os.listdir(os.path.join(reference, "tests"))):
        if f.endswith(".py"):
            shutil.copyfile(os.path.join(reference, "tests", f), os.path.join(tests, f))
    for d, subdirs, _ in os.walk(dest):
        if "__pycache__" in subdirs:
            shutil.rmtree(os.path.join(d, "__pycache__"))
    return dest


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("DS_REFERENCE"),
                    help="root of the reference checkout (or set DS_REFERENCE)")
    a = ap.parse_args()
    if not a.reference:
        ap.error("give --reference PATH (or set DS_REFERENCE)")
    print(stage(a.reference))
