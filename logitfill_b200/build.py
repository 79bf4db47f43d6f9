"""Build the sm_100a C-ABI library in-tree (``logitfill_b200/_lib/``).

    python -m logitfill_b200.build          # or __graft_entry__.build()

nvcc cross-compiles for B200 without a GPU.  The shared library links the
CUDA runtime statically and exports only the ``lf_*`` symbols declared in
``include/logitfill_b200.h``.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OUT_DIR = PKG / "_lib"
LIB_NAME = "liblogitfill_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found; the CUDA 12.9 toolkit is required to build logitfill_b200")
    return found


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def build(verbose: bool = False, force: bool = False) -> Path:
    OUT_DIR.mkdir(exist_ok=True)
    out = OUT_DIR / LIB_NAME
    srcs = sources()
    deps = srcs + sorted(CSRC.glob("*.cuh")) + [ROOT / "include" / "logitfill_b200.h", Path(__file__)]
    if not force and out.exists() and all(out.stat().st_mtime >= d.stat().st_mtime for d in deps):
        return out
    build_dir = OUT_DIR / "obj"
    build_dir.mkdir(exist_ok=True)
    common = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden",
              "-I", str(ROOT / "include"), "-I", str(CSRC), "--expt-relaxed-constexpr"]
    objs = []
    procs = []
    for src in srcs:
        obj = build_dir / (src.stem + ".o")
        cmd = common + ["-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
        objs.append(obj)
    failed = []
    for src, proc in procs:
        log = proc.communicate()[0].decode()
        if proc.returncode != 0:
            failed.append(f"{src.name}:\n{log}")
        elif verbose and log.strip():
            print(log)
    if failed:
        raise RuntimeError("nvcc failed:\n" + "\n".join(failed))
    tmp = out.with_suffix(".so.tmp")
    link = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-cudart", "static"]
    if verbose:
        print(" ".join(link), flush=True)
    subprocess.run(link, check=True)
    os.replace(tmp, out)
    return out


if __name__ == "__main__":
    path = build(verbose="-v" in sys.argv, force="-f" in sys.argv)
    print(path)
