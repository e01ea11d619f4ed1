"""Build the in-tree CUDA library (sm_100a) with nvcc.

    python -m xinfer_b200.build [--force]

Produces xinfer_b200/libxinfer_b200.so from xinfer_b200/csrc/*.cu. The library is plain C ABI
(include/xinfer_b200.h) linked against the CUDA runtime only; torch is not needed to build it.
"""

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
OUT = PKG / "libxinfer_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
         "--expt-relaxed-constexpr", "-Xptxas", "-v"]


def nvcc():
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found")
    return path


def sources():
    return sorted(CSRC.glob("*.cu"))


def headers():
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def up_to_date():
    if not OUT.exists():
        return False
    t = OUT.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in sources() + headers())


def build(force=False, verbose=False):
    if not force and up_to_date():
        return OUT
    cmd = [nvcc(), *ARCH, *FLAGS, f"-I{INCLUDE}", f"-I{CSRC}", "-o", str(OUT) + ".tmp",
           *map(str, sources())]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    log = proc.stdout + proc.stderr
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed:\n{' '.join(cmd)}\n{log}")
    os.replace(str(OUT) + ".tmp", OUT)
    (PKG / "build_ptxas.log").write_text(log)
    if verbose:
        print(log)
    return OUT


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args()
    out = build(force=args.force, verbose=args.verbose)
    print(out)


if __name__ == "__main__":
    sys.exit(main())
