"""Build libb200moe.so in-tree for sm_100a.

    python sglang-restomod_b200/build.py [--force]

Every .cu file under csrc/ is compiled with nvcc for ``sm_100a`` only and
linked into ``sglang_restomod_b200/libb200moe.so`` (static CUDA runtime, no
torch dependency). The build is skipped when the library is newer than every
source and header.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
OUT = HERE / "sglang_restomod_b200" / "libb200moe.so"
OBJ_DIR = HERE / "_build"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise FileNotFoundError("nvcc not found (set NVCC or put CUDA's bin on PATH)")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _inputs() -> list[Path]:
    return sources() + sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def up_to_date() -> bool:
    if not OUT.exists():
        return False
    built = OUT.stat().st_mtime
    return all(p.stat().st_mtime <= built for p in _inputs())


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile (if stale) and return the path of libb200moe.so."""
    if not force and up_to_date():
        return OUT
    nvcc = _nvcc()
    OBJ_DIR.mkdir(exist_ok=True)
    objs = []
    procs = []
    for src in sources():
        obj = OBJ_DIR / (src.stem + ".o")
        cmd = [nvcc, *ARCH, *FLAGS, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
        objs.append(obj)
    failed = []
    for src, proc in procs:
        out, _ = proc.communicate()
        if proc.returncode != 0:
            failed.append(f"{src.name}:\n{out.decode(errors='replace')}")
        elif verbose and out:
            print(out.decode(errors="replace"))
    if failed:
        raise RuntimeError("nvcc failed:\n" + "\n".join(failed))
    tmp = OUT.with_suffix(".so.tmp")
    link = [nvcc, *ARCH, "-shared", "-o", str(tmp), *map(str, objs)]
    subprocess.run(link, check=True)
    os.replace(tmp, OUT)
    return OUT


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args()
    path = build(force=args.force, verbose=args.verbose)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
