"""Install the unmodified reference implementation (FlashUMA) into ``baseline/_ref``.

    python baseline/install_reference.py <path of the reference source tree>
    FLASHUMA_REFERENCE=<path> python baseline/install_reference.py

``bench.py`` times the reference's own Triton path on the GPU from ``baseline/_ref``
(git-ignored; it travels with the working tree to the GPU box). The recipe first tries
the standard offline install

    python -m pip install --no-index --no-build-isolation --find-links /opt/wheelhouse \
        --target baseline/_ref <reference>

The reference is a plain source tree with neither ``setup.py`` nor ``pyproject.toml``, so
pip refuses it ("not installable"). The recipe then does what an install of a pure-Python
tree amounts to: it copies the reference's importable sources (``model.py``, ``wrapper.py``,
``ops/*.py``) byte for byte into ``baseline/_ref`` and writes ``INSTALLED.txt`` with the
outcome and the SHA-256 of every copied file. Nothing is edited.
"""
from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
TARGET = os.path.join(HERE, "_ref")
SOURCES = ["model.py", "wrapper.py", "ops/__init__.py", "ops/constants.py", "ops/geom.py", "ops/gather.py",
           "ops/gating.py", "ops/scatter.py", "ops/ln_silu.py"]


def main() -> int:
    src = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("FLASHUMA_REFERENCE")
    if not src or not os.path.isfile(os.path.join(src, "ops", "gather.py")):
        print("usage: install_reference.py <reference source tree> (or set FLASHUMA_REFERENCE)", file=sys.stderr)
        return 2
    os.makedirs(TARGET, exist_ok=True)
    pip = subprocess.run([sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation",
                          "--find-links", "/opt/wheelhouse", "--target", TARGET, src],
                         capture_output=True, text=True)
    lines = [f"pip install --target {TARGET}: rc {pip.returncode}"]
    lines += ["  " + ln for ln in (pip.stdout + pip.stderr).strip().splitlines()[-3:]]
    if pip.returncode != 0:
        lines.append("fallback: byte-for-byte copy of the reference's importable sources")
        for rel in SOURCES:
            s = os.path.join(src, rel)
            if not os.path.exists(s):
                if rel == "ops/__init__.py":
                    continue   # a namespace package is fine
                print(f"missing reference file {rel}", file=sys.stderr)
                return 1
            d = os.path.join(TARGET, rel)
            os.makedirs(os.path.dirname(d), exist_ok=True)
            shutil.copyfile(s, d)
            lines.append(f"  {rel} sha256 {hashlib.sha256(open(d, 'rb').read()).hexdigest()}")
    with open(os.path.join(TARGET, "INSTALLED.txt"), "w") as f:
        f.write("\n".join(lines) + "\n")
    print("\n".join(lines))
    return 0


if __name__ == "__main__":
    sys.exit(main())
