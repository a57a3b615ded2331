"""Build recipe for the oracle's C restatement (oracle/_build/liboracle.so).

Test infrastructure only: gcc -O2 -fopenmp on a8w4_oracle.c. The output directory
oracle/_build/ is not committed.
"""
from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

ORACLE_DIR = Path(__file__).resolve().parent
SRC = ORACLE_DIR / "a8w4_oracle.c"
OUT = ORACLE_DIR / "_build" / "liboracle.so"


def build_oracle(force: bool = False) -> Path:
    if OUT.exists() and not force and OUT.stat().st_mtime >= SRC.stat().st_mtime:
        return OUT
    OUT.parent.mkdir(parents=True, exist_ok=True)
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        raise RuntimeError("no C compiler found for the oracle")
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [cc, "-O2", "-fPIC", "-shared", "-fopenmp", "-o", str(tmp), str(SRC), "-lm"]
    subprocess.run(cmd, check=True)
    tmp.replace(OUT)
    return OUT


if __name__ == "__main__":
    print(build_oracle(force=True))
