"""Builds the CPU oracle (test infrastructure) into oracle/_build/liboracle.so.

The oracle is compiled with -ffp-contract=off so that no multiply-add is fused
implicitly; its floating-point specification is documented in omni_oracle.c.
"""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

ROOT = Path(__file__).resolve().parent
SRC = ROOT / "omni_oracle.c"
OUT = ROOT / "_build" / "liboracle.so"


def build() -> Path:
    OUT.parent.mkdir(exist_ok=True)
    if OUT.exists() and OUT.stat().st_mtime >= SRC.stat().st_mtime:
        return OUT
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        raise RuntimeError("no C compiler found for the oracle")
    cmd = [cc, "-O2", "-std=c11", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared", "-Wall",
           "-o", str(OUT), str(SRC), "-lm"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{proc.stderr}")
    return OUT


if __name__ == "__main__":
    print(build())
