"""Install the reference (djsaunde/spikegpt-myelin) into ``baseline/_ref``.

    python baseline/install_ref.py [--reference /path/to/spikegpt-myelin]

``baseline/_ref`` is git-ignored; it travels to GPU boxes with the working tree
so the reference's own Python code can run there (its Triton WKV kernels as the
incumbent, its CPU ``weighted_key_value`` as the reference arm of bench.py, and
its model blocks through this package's drop-in). Nothing under ``baseline/``
is imported by the product path.

First the standard offline install is tried:

    pip install --no-index --no-build-isolation --find-links /opt/wheelhouse \
        --target baseline/_ref --no-deps <reference>

The reference builds with ``uv_build`` (pyproject ``[build-system]``), which is
not in the offline wheelhouse, so that command fails here. The package is pure
Python (``src/spikegpt``, module-root ``src`` in ``[tool.uv.build-backend]``),
so the fallback places exactly what its wheel would contain: the files of
``src/spikegpt`` under ``baseline/_ref/spikegpt``. Its dependency ``myelin`` is
not installable offline either; tests and bench.py put the test-only stand-in
``tests/golden/_myelin_shim`` on ``sys.path`` instead.

The outcome is written to ``baseline/_ref/INSTALL.txt``.
"""

from __future__ import annotations

import argparse
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
TARGET = HERE / "_ref"


def install(reference: Path, target: Path = TARGET) -> str:
    if not (reference / "src" / "spikegpt" / "language.py").exists():
        raise SystemExit(f"{reference} is not a spikegpt-myelin checkout")
    target.mkdir(parents=True, exist_ok=True)
    cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation",
           "--find-links", "/opt/wheelhouse", "--target", str(target), "--no-deps", "--upgrade",
           str(reference)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode == 0 and (target / "spikegpt" / "language.py").exists():
        outcome = "pip install succeeded"
    else:
        tail = (r.stderr or r.stdout).strip().splitlines()[-1:] or ["(no output)"]
        dst = target / "spikegpt"
        if dst.exists():
            shutil.rmtree(dst)
        shutil.copytree(reference / "src" / "spikegpt", dst,
                        ignore=shutil.ignore_patterns("__pycache__", "*.pyc"))
        outcome = ("pip install failed (" + tail[0].strip() + "); placed the pure-Python package "
                   "src/spikegpt as its wheel would")
    (target / "INSTALL.txt").write_text(outcome + "\n")
    return outcome


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default="/root/reference")
    args = ap.parse_args()
    print(install(Path(args.reference)))


if __name__ == "__main__":
    main()
