"""Build ``libaltxs_b200.so`` (the C-ABI library) in-tree for sm_100a.

    python -m altxs_b200.build            # nvcc all csrc/*.cu into one .so

The library links only the CUDA runtime (no torch), so any host language can
load it.  The built ``.so`` sits next to this file and travels with the tree.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
LIB = HERE / "libaltxs_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-shared", "--expt-relaxed-constexpr"]


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = sources() + sorted(CSRC.glob("*.cuh")) + [HERE.parent / "include" / "altxs_b200.h"]
    return any(p.stat().st_mtime > t for p in deps)


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found")
    return cand


def build(force: bool = False, verbose: bool = False, jobs: int | None = None) -> Path:
    """Compile each ``csrc/*.cu`` to an object in parallel, then link the .so."""
    if not force and not _stale():
        return LIB
    obj_dir = HERE / "_build"
    obj_dir.mkdir(exist_ok=True)
    compile_flags = [f for f in FLAGS if f != "-shared"]
    cmds = []
    for src in sources():
        cmd = [nvcc(), *ARCH, *compile_flags, "-c", "-o", str(obj_dir / (src.stem + ".o")), str(src)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd), file=sys.stderr)
        cmds.append(cmd)
    jobs = jobs or max(1, min(len(cmds), os.cpu_count() or 1))
    with ThreadPoolExecutor(jobs) as ex:
        procs = list(ex.map(lambda c: subprocess.run(c, cwd=str(CSRC)), cmds))
    bad = [c[-1] for c, p in zip(cmds, procs) if p.returncode]
    if bad:
        raise RuntimeError(f"nvcc failed on {', '.join(bad)}")
    tmp = LIB.with_suffix(".so.tmp")
    objs = [str(obj_dir / (src.stem + ".o")) for src in sources()]
    subprocess.run([nvcc(), *ARCH, "-shared", "-o", str(tmp), *objs], check=True, cwd=str(CSRC))
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
