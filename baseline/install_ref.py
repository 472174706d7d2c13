"""Install the reference package (acrosley/marathon) into ``baseline/_ref``.

The reference arm of ``bench.py`` and the gap-fill hand-off tests import the
reference's own, unmodified ``marathon`` package from ``baseline/_ref``
(git-ignored: it is an install, not part of this repository's source).

The reference is pure Python.  Its wheel is built with hatchling, which the
offline wheelhouse does not carry, so the contract's install command

    pip install --no-index --no-build-isolation --find-links <wheelhouse> \\
        --target baseline/_ref <reference checkout>

stops before installing anything ("No module named 'hatchling'").  This recipe
tries that command first and, when it fails, writes what it would have
written: the package directory ``src/marathon`` copied byte for byte to
``baseline/_ref/marathon`` (the layout ``pip install --target`` produces for a
pure-Python package), plus ``baseline/_ref/INSTALL.txt`` naming the source
and a SHA-256 of every copied file.

    python baseline/install_ref.py <reference checkout> [--wheelhouse DIR]
"""

from __future__ import annotations

import argparse
import hashlib
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
TARGET = HERE / "_ref"


def _pip(checkout: Path, wheelhouse: Path) -> tuple[bool, str]:
    cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation",
           "--find-links", str(wheelhouse), "--target", str(TARGET), str(checkout)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    tail = (r.stdout + r.stderr).strip().splitlines()[-1:] or [""]
    return r.returncode == 0 and (TARGET / "marathon").is_dir(), tail[0]


def _copy(checkout: Path) -> list[str]:
    src = checkout / "src" / "marathon"
    if not (src / "__init__.py").is_file():
        raise SystemExit(f"{checkout} has no src/marathon package")
    dst = TARGET / "marathon"
    if dst.exists():
        shutil.rmtree(dst)
    shutil.copytree(src, dst, ignore=shutil.ignore_patterns("__pycache__", "*.pyc"))
    lines = []
    for f in sorted(dst.rglob("*.py")):
        digest = hashlib.sha256(f.read_bytes()).hexdigest()
        lines.append(f"{digest}  {f.relative_to(TARGET)}")
    return lines


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("checkout", type=Path, help="the reference checkout (holds src/marathon)")
    ap.add_argument("--wheelhouse", type=Path, default=None,
                    help="offline wheelhouse for the pip attempt (omitted: copy directly)")
    args = ap.parse_args(argv)
    TARGET.mkdir(parents=True, exist_ok=True)
    ok, why = (_pip(args.checkout, args.wheelhouse) if args.wheelhouse is not None
               else (False, "no wheelhouse given"))
    if ok:
        how = "pip install --target (wheel built from the checkout)"
        files = []
    else:
        how = f"copy of src/marathon (pip install failed: {why})"
        files = _copy(args.checkout)
    (TARGET / "INSTALL.txt").write_text(
        f"source: {args.checkout}\nmethod: {how}\n" + "".join(f"{x}\n" for x in files))
    print(f"baseline/_ref/marathon installed by {how}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
