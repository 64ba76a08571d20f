"""Install the unmodified reference package (mESmaC/spalmer) into ``baseline/_ref``.

Test/benchmark infrastructure only: ``bench.py --impl reference`` (and the
``cpu_baseline`` leg of the default arm) time the reference's own
``MicroExpertChannelMixer.forward`` on the host cores from this install.  The
product path never imports it.

The reference declares ``hatchling`` as its build backend, which the offline
wheelhouse does not carry.  The recipe therefore copies the reference tree to a
scratch folder under /tmp, replaces only the ``[build-system]`` and
``[tool.hatch.*]`` tables of that copy's ``pyproject.toml`` with the
setuptools equivalent (package ``spalmer`` under ``src/``), and runs

    pip install --no-index --no-build-isolation --no-deps --find-links /opt/wheelhouse \
        --target baseline/_ref <copy>

``--no-deps``: the reference's only other dependency, ``zstandard``, is used by
its data pipeline, not by the expert layer, and is not in the wheelhouse.  The
Python sources installed are the reference's own, byte for byte (checked
below against the source tree).

    python oracle/install_ref.py --reference PATH    (or $SPALMER_REFERENCE)

PATH is the reference project's root (the folder holding ``pyproject.toml``
and ``src/spalmer``).
"""

from __future__ import annotations

import argparse
import filecmp
import os
import re
import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
TARGET = ROOT / "baseline" / "_ref"

SETUPTOOLS_TABLES = """[build-system]
requires = ["setuptools"]
build-backend = "setuptools.build_meta"

[tool.setuptools.packages.find]
where = ["src"]
"""


def _rewrite_pyproject(text: str) -> str:
    # Drop [build-system] and every [tool.hatch...] table; keep the rest as it is.
    out, skip = [], False
    for line in text.splitlines():
        header = re.match(r"^\[([^\]]+)\]\s*$", line)
        if header:
            name = header.group(1).strip()
            skip = name == "build-system" or name.startswith("tool.hatch")
        if not skip:
            out.append(line)
    return "\n".join(out).rstrip() + "\n\n" + SETUPTOOLS_TABLES


def install(reference: Path, target: Path = TARGET) -> Path:
    reference = reference.resolve()
    if not (reference / "src" / "spalmer" / "experts" / "mixer.py").exists():
        raise FileNotFoundError(f"no reference package under {reference}")
    with tempfile.TemporaryDirectory(prefix="spalmer_ref_") as tmp:
        copy = Path(tmp) / "spalmer"
        shutil.copytree(reference, copy, ignore=shutil.ignore_patterns(".git", "__pycache__", "tests", "docs"))
        py = copy / "pyproject.toml"
        py.write_text(_rewrite_pyproject(py.read_text()))
        if target.exists():
            shutil.rmtree(target)
        target.parent.mkdir(parents=True, exist_ok=True)
        cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--no-deps",
               "--find-links", "/opt/wheelhouse", "--target", str(target), str(copy)]
        subprocess.run(cmd, check=True, stdout=subprocess.DEVNULL)
    # The installed sources must be the reference's own.
    src = reference / "src" / "spalmer"
    for path in src.rglob("*.py"):
        installed = target / "spalmer" / path.relative_to(src)
        if not installed.exists() or not filecmp.cmp(path, installed, shallow=False):
            raise RuntimeError(f"installed file differs from the reference: {installed}")
    return target


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--reference", default=os.environ.get("SPALMER_REFERENCE"))
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference PATH or set SPALMER_REFERENCE")
    print(install(Path(args.reference)))


if __name__ == "__main__":
    main()
