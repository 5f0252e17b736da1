"""Ahead-of-time build of the CUDA library ``cresso_b200/_C/libcresso_b200.so``.

Compiles every ``csrc/*.cu`` for sm_100a with nvcc (no JIT, no torch
extension machinery) and links one shared library with a plain C ABI
(``include/cresso_b200.h``).  Run ``python -m cresso_b200.build``.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
OUT_DIR = PKG / "_C"
LIB = OUT_DIR / "libcresso_b200.so"
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
              "-Xcompiler", "-fvisibility=hidden", "-Xptxas", "-warn-spills"]


def nvcc() -> str:
    for cand in (os.environ.get("CUDACXX"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; the CUDA library is built ahead of time with nvcc")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    deps = [src] + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + [PKG.parent / "include" / "cresso_b200.h"]
    return any(d.stat().st_mtime > obj.stat().st_mtime for d in deps)


def build(verbose: bool = False, force: bool = False, extra: list[str] | None = None) -> Path:
    OUT_DIR.mkdir(exist_ok=True)
    obj_dir = OUT_DIR / "obj"
    obj_dir.mkdir(exist_ok=True)
    cc = nvcc()
    extra = list(extra or [])
    jobs = []
    for src in sources():
        obj = obj_dir / (src.stem + ".o")
        if force or _stale(obj, src):
            cmd = [cc, *ARCH_FLAGS, *NVCC_FLAGS, *extra, "-I", str(PKG.parent / "include"), "-c", str(src), "-o", str(obj)]
            jobs.append((src, cmd))
    def run(job):
        src, cmd = job
        r = subprocess.run(cmd, capture_output=True, text=True)
        return src, cmd, r
    with cf.ThreadPoolExecutor(max_workers=max(1, min(8, os.cpu_count() or 1))) as ex:
        for src, cmd, r in ex.map(run, jobs):
            if verbose or r.returncode != 0:
                sys.stderr.write(f"$ {' '.join(cmd)}\n{r.stdout}{r.stderr}")
            if r.returncode != 0:
                raise RuntimeError(f"nvcc failed on {src.name}")
    objs = [str(obj_dir / (s.stem + ".o")) for s in sources()]
    if force or jobs or not LIB.exists():
        cmd = [cc, *ARCH_FLAGS, "-shared", "-o", str(LIB), *objs, "-cudart", "static", "-Xcompiler", "-fPIC"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if verbose or r.returncode != 0:
            sys.stderr.write(f"$ {' '.join(cmd)}\n{r.stdout}{r.stderr}")
        if r.returncode != 0:
            raise RuntimeError("nvcc link of libcresso_b200.so failed")
    return LIB


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, force="-f" in sys.argv)
    print(LIB)
