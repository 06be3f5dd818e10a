"""Build the sm_100a shared library ``_lib/libgranule_b200.so`` with nvcc.

Every ``csrc/*.cu`` file is compiled for ``compute_100a``/``sm_100a`` and linked
into one shared object that exports the C ABI declared in
``include/granule_b200.h``.  The library links the shared CUDA runtime
(``libcudart.so.12``), so inside a PyTorch process it shares torch's runtime
instance; outside one it finds the toolkit's copy through its rpath.

Run ``python -m granulelayer_b200.build`` (or ``__graft_entry__.build()``).
Objects are rebuilt when a source or header is newer than the library; the
sources compile in parallel (one nvcc per core).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB_DIR = PKG / "_lib"
LIB = LIB_DIR / "libgranule_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))


def nvcc() -> str:
    cand = CUDA_HOME / "bin" / "nvcc"
    if cand.exists():
        return str(cand)
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found (set CUDA_HOME)")
    return found


def sources():
    return sorted(CSRC.glob("*.cu"))


def _stale(out: Path, deps) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(p.stat().st_mtime > t for p in deps)


def build(verbose: bool = False, force: bool = False) -> Path:
    LIB_DIR.mkdir(exist_ok=True)
    obj_dir = LIB_DIR / "obj"
    obj_dir.mkdir(exist_ok=True)
    headers = list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    flags = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", f"-I{INCLUDE}", f"-I{CSRC}", *ARCH]
    objs, cmds = [], []
    for src in sources():
        obj = obj_dir / (src.stem + ".o")
        objs.append(obj)
        if force or _stale(obj, [src, *headers]):
            cmds.append([nvcc(), "-c", str(src), "-o", str(obj), *flags])

    def compile_one(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)

    if cmds:
        with ThreadPoolExecutor(max_workers=max(1, min(len(cmds), os.cpu_count() or 1))) as ex:
            list(ex.map(compile_one, cmds))
    if force or _stale(LIB, objs):
        cmd = [nvcc(), "-shared", "-o", str(LIB), *map(str, objs), *ARCH, "-cudart", "shared",
               "-Xlinker", f"-rpath={CUDA_HOME / 'lib64'}"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(verbose=True, force="--force" in sys.argv)
    print(LIB)
