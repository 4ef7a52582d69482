"""Build the in-tree C-ABI library ``d2sd_b200/libd2sd.so`` for sm_100a.

Every CUDA source is compiled with ``nvcc -gencode arch=compute_100a,code=sm_100a
-lineinfo``; the host sources go through nvcc as well, and the objects are linked
into one shared library with a static CUDA runtime. Cross-compiles without a
GPU. Rebuilds only what changed (source or header newer than its object).

    python -m d2sd_b200.build            # build
    python -m d2sd_b200.build --force    # rebuild everything
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libd2sd.so"
INCLUDE = PKG.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
          "--expt-relaxed-constexpr", f"-I{INCLUDE}"]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build d2sd")
    return path


def sources() -> list[Path]:
    return sorted(p for p in CSRC.iterdir() if p.suffix in (".cu", ".cpp"))


def headers() -> list[Path]:
    hs = [p for p in CSRC.iterdir() if p.suffix in (".cuh", ".h")]
    hs += list(INCLUDE.glob("*.h"))
    return hs


def _compile(src: Path, obj: Path, verbose: bool) -> None:
    cmd = [nvcc(), *ARCH, *COMMON, "-c", str(src), "-o", str(obj)]
    if src.suffix == ".cu":
        cmd += ["-Xptxas", "-v"] if verbose else []
    else:
        cmd = [nvcc(), *ARCH, *COMMON, "-x", "c++", "-c", str(src), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    if verbose and res.stderr:
        sys.stderr.write(res.stderr)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile changed sources and relink ``libd2sd.so``; returns its path."""
    BUILD.mkdir(exist_ok=True)
    newest_header = max((h.stat().st_mtime for h in headers()), default=0.0)
    jobs = []
    objs = []
    for src in sources():
        obj = BUILD / (src.name + ".o")
        objs.append(obj)
        stale = force or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime,
                                                                       newest_header)
        if stale:
            jobs.append((src, obj))
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(8, len(jobs))) as ex:
            list(ex.map(lambda j: _compile(j[0], j[1], verbose), jobs))
    if jobs or force or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed: {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/smem usage")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))


if __name__ == "__main__":
    main()
