"""Install the reference's ``_int4`` package into ``baseline/_ref`` -- BASELINE INFRASTRUCTURE.

``bench.py --impl reference`` (and the CPU-baseline leg of the default run)
time the reference's own CPU implementation of the path,
``_int4.eager.convrot_w4a4_linear`` (its forward on a host without the HIP
kernel), imported from ``baseline/_ref``. That directory is not part of the
repository's history; this script makes it from a reference checkout, offline:

    python oracle/ref_install.py [--reference <checkout>]

It runs ``pip install --no-index --no-deps --no-build-isolation --target
baseline/_ref`` on a copy of the checkout in a temporary directory. The copy's
pyproject.toml gets one addition: the package list ``["_int4"]``. The
reference's pyproject declares no package list, and setuptools refuses its
flat layout (several top-level modules) without one. No source file is changed.
The installed ``_int4`` imports without ROCm; only its HIP entry points need a
gfx12 device, and the eager path needs none.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import tempfile

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TARGET = os.path.join(ROOT, "baseline", "_ref")
DEFAULT_REFERENCE = os.environ.get("CONVROT_REFERENCE", "/root/reference")
PACKAGE_TABLE = '\n[tool.setuptools]\npackages = ["_int4"]\n\n[tool.setuptools.package-data]\n_int4 = ["*.hip"]\n'


def installed() -> bool:
    return os.path.exists(os.path.join(TARGET, "_int4", "eager.py"))


def install(reference: str = DEFAULT_REFERENCE, quiet: bool = True) -> bool:
    """Install when missing; True when ``baseline/_ref/_int4`` is present afterwards."""
    if installed():
        return True
    if not os.path.exists(os.path.join(reference, "_int4", "eager.py")):
        return False
    with tempfile.TemporaryDirectory() as tmp:
        src = os.path.join(tmp, "reference")
        shutil.copytree(reference, src, ignore=shutil.ignore_patterns(".git", "__pycache__"))
        with open(os.path.join(src, "pyproject.toml"), "a") as f:
            f.write(PACKAGE_TABLE)
        cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-deps", "--no-build-isolation",
               "--target", TARGET, src]
        wheels = "/opt/wheelhouse"
        if os.path.isdir(wheels):
            cmd[4:4] = ["--find-links", wheels]
        cp = subprocess.run(cmd, capture_output=True, text=True)
        if cp.returncode != 0 and not quiet:
            print(cp.stdout[-2000:], cp.stderr[-2000:], file=sys.stderr)
    return installed()


if __name__ == "__main__":
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--reference", default=DEFAULT_REFERENCE)
    a = ap.parse_args()
    ok = install(a.reference, quiet=False)
    print("baseline/_ref/_int4:", "installed" if ok else "not installed")
    sys.exit(0 if ok else 1)
