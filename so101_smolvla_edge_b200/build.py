"""Build libso101_b200.so in-tree with nvcc for sm_100a.

    python -m so101_smolvla_edge_b200.build [--force] [-v]

Each .cu under csrc/ compiles to an object in parallel, then one shared library links them with
the static CUDA runtime. The result lands in `so101_smolvla_edge_b200/lib/`, next to the package,
so it travels with the source tree; nothing is installed elsewhere.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
OUT_DIR = PKG / "lib"
LIB = OUT_DIR / "libso101_b200.so"
BUILD_DIR = PKG.parent / "_build" / "obj"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
         "-Xcompiler", "-fvisibility=hidden"]  # fmt: skip


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put CUDA's bin on PATH")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    """Compile what changed and link the library; return its path."""
    headers = list(CSRC.glob("*.cuh")) + list((PKG.parent / "include").glob("*.h"))
    srcs = sources()
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    cc = nvcc()
    jobs = []
    for src in srcs:
        obj = BUILD_DIR / (src.stem + ".o")
        if force or ptxas_info or _stale(obj, [src, *headers]):
            cmd = [cc, *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
            if ptxas_info:
                cmd += ["-Xptxas", "-v"]
            jobs.append((src, cmd))

    def run(job):
        src, cmd = job
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        return src, r

    with ThreadPoolExecutor(max_workers=min(8, max(1, len(jobs)))) as ex:
        results = list(ex.map(run, jobs))
    failed = [(s, r) for s, r in results if r.returncode != 0]
    for s, r in results:
        if (verbose or ptxas_info or r.returncode) and (r.stdout or r.stderr):
            print(f"--- {s.name}\n{r.stdout}{r.stderr}", file=sys.stderr)
    if failed:
        raise RuntimeError(f"nvcc failed for {[s.name for s, _ in failed]}")
    objs = [BUILD_DIR / (s.stem + ".o") for s in srcs]
    if force or jobs or _stale(LIB, objs):
        cmd = [cc, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-cudart", "static"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode:
            raise RuntimeError(f"link failed:\n{r.stdout}{r.stderr}")
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers/spills per kernel")
    a = ap.parse_args()
    print(build(a.force, a.verbose, a.ptxas_info))


if __name__ == "__main__":
    main()
