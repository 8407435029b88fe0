"""In-tree build of the TurboCider CUDA backend: libturbocider_cuda.so.

Compiles every source under csrc/ for sm_100a only (``-gencode
arch=compute_100a,code=sm_100a``) with nvcc, in parallel, and links one
shared library next to this file so that it travels with the repository.
No JIT cache is used.  Run ``python -m turbocider_b200.build``.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
OUT = HERE / "libturbocider_cuda.so"
# The bounds-checked variant (-DTC_BOUNDS_CHECK): every output store, weight
# chunk address and decode target offset is checked, an index outside sets
# TC_STATUS_BOUNDS instead of faulting.  The substitute for compute-sanitizer
# in the GPU tests; loaded when TURBOCIDER_CHECKED=1.
OUT_CHECKED = HERE / "libturbocider_cuda_checked.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
          "--expt-relaxed-constexpr", "-I", str(HERE.parent / "include")]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found: the CUDA backend cannot be built")
    return path


def sources() -> list[Path]:
    return sorted(p for p in CSRC.iterdir() if p.suffix in (".cu", ".cpp"))


def _compile(src: Path, obj_dir: Path, defines: list[str], verbose: bool) -> Path:
    obj = obj_dir / (src.stem + ".o")
    deps = [src] + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list((HERE.parent / "include").glob("*.h"))
    if obj.exists() and obj.stat().st_mtime >= max(d.stat().st_mtime for d in deps):
        return obj
    cmd = [nvcc(), *ARCH, *COMMON, *defines, "-c", str(src), "-o", str(obj)]
    if src.suffix == ".cu" and verbose:
        cmd += ["-Xptxas", "-v"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stderr}")
    if verbose and res.stderr:
        print(res.stderr, file=sys.stderr)
    return obj


def build(verbose: bool = False, checked: bool | None = None) -> Path:
    """Build the library (and, unless checked is False, its bounds-checked
    variant); returns the path of the normal library (checked=True: of the
    checked one only)."""
    variants = [(OUT, HERE / "_build", [])] if checked is not True else []
    if checked is not False:
        variants.append((OUT_CHECKED, HERE / "_build_checked", ["-DTC_BOUNDS_CHECK"]))
    srcs = sources()
    jobs = []
    for out, obj_dir, defines in variants:
        obj_dir.mkdir(exist_ok=True)
        jobs += [(src, obj_dir, defines) for src in srcs]
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as pool:
        objs = list(pool.map(lambda j: _compile(j[0], j[1], j[2], verbose), jobs))
    for i, (out, obj_dir, defines) in enumerate(variants):
        mine = objs[i * len(srcs):(i + 1) * len(srcs)]
        if out.exists() and out.stat().st_mtime >= max(o.stat().st_mtime for o in mine):
            continue
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(out), *map(str, mine), "-lpthread"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stderr}")
    return variants[0][0]


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
