"""Build the in-tree libraries.

    python -m xinfer_b200.build [--force]

  * xinfer_b200/libxinfer_b200.so from xinfer_b200/csrc/*.cu with nvcc for sm_100a (one object per
    translation unit, compiled in parallel): the plain C ABI of include/xinfer_b200.h, linked
    against the CUDA runtime only (no torch);
  * xinfer_b200/libxinfer_b200_ops.so from xinfer_b200/csrc/torch_ops.cpp with the host C++
    compiler: the xinfer::qwen3_decode_step / qwen35_decode_step torch operators and their
    AOTInductor C shims, linked against libtorch and libxinfer_b200.so (found next to it).
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
OPS_SRC = CSRC / "torch_ops.cpp"
OPS_OUT = PKG / "libxinfer_b200_ops.so"
BUILD_DIR = PKG / "_build"  # object files (not committed)

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


FLAGS_CU = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr", "-Xptxas", "-v"]


def nvcc():
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found")
    return path


def sources():
    return sorted(CSRC.glob("*.cu"))


def torch_flags():
    import torch
    from torch.utils import cpp_extension

    inc = cpp_extension.include_paths(device_type="cuda")
    lib = cpp_extension.library_paths(device_type="cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    flags = [f"-I{p}" for p in inc] + [f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_API_INCLUDE_EXTENSION_H"]
    libs = [f"-L{p}" for p in lib] + [f"-Wl,-rpath,{p}" for p in lib]
    libs += ["-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-lc10_cuda", "-L/usr/local/cuda/lib64",
             "-lcudart"]
    return flags, libs


def build_ops(force=False):
    """The torch operator library (host C++ only; the kernels stay in libxinfer_b200.so)."""
    if not force and OPS_OUT.exists() and OPS_OUT.stat().st_mtime >= max(
            OPS_SRC.stat().st_mtime, OUT.stat().st_mtime, (INCLUDE / "xinfer_b200.h").stat().st_mtime):
        return OPS_OUT
    flags, libs = torch_flags()
    cxx = shutil.which("g++") or "c++"
    cmd = [cxx, "-O2", "-std=c++17", "-fPIC", "-shared", *flags, f"-I{INCLUDE}", "-o", str(OPS_OUT) + ".tmp",
           str(OPS_SRC), f"-L{PKG}", "-lxinfer_b200", "-Wl,-rpath,$ORIGIN", *libs]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"g++ failed:\n{' '.join(cmd)}\n{proc.stdout}{proc.stderr}")
    os.replace(str(OPS_OUT) + ".tmp", OPS_OUT)
    return OPS_OUT


def headers():
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def up_to_date():
    if not OUT.exists():
        return False
    t = OUT.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in sources() + headers())


def _compile(src, obj, force):
    """One translation unit to an object file (skipped when the object is newer than it and every
    header); returns the ptxas report."""
    newest = max([src.stat().st_mtime] + [h.stat().st_mtime for h in headers()])
    if not force and obj.exists() and obj.stat().st_mtime >= newest:
        return ""
    cmd = [nvcc(), *ARCH, *FLAGS_CU, f"-I{INCLUDE}", f"-I{CSRC}", "-c", "-o", str(obj) + ".tmp",
           str(src)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    log = proc.stdout + proc.stderr
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed:\n{' '.join(cmd)}\n{log}")
    os.replace(str(obj) + ".tmp", obj)
    return f"== {src.name}\n{log}"


def build(force=False, verbose=False):
    if not force and up_to_date():
        return OUT
    from concurrent.futures import ThreadPoolExecutor

    BUILD_DIR.mkdir(exist_ok=True)
    srcs = sources()
    objs = [BUILD_DIR / (s.stem + ".o") for s in srcs]
    with ThreadPoolExecutor(max_workers=max(1, min(len(srcs), os.cpu_count() or 1))) as pool:
        logs = list(pool.map(lambda so: _compile(so[0], so[1], force), zip(srcs, objs)))
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(OUT) + ".tmp", *map(str, objs)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc link failed:\n{' '.join(cmd)}\n{proc.stdout}{proc.stderr}")
    os.replace(str(OUT) + ".tmp", OUT)
    log = "".join(logs)
    if log:
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
    print(build_ops(force=args.force))


if __name__ == "__main__":
    sys.exit(main())
