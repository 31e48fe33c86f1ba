"""Build libflexattn.so in-tree with nvcc for sm_100a.

    python pallas-flexattn_b200/build.py [--force] [--debug]

Each csrc/*.cu is compiled to an object under _build/ (skipped when newer than
its sources and headers), then linked into pallas_flexattn/libflexattn.so, the
library the Python package loads.  No GPU is needed to build.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
REPO = PKG_ROOT.parent
CSRC = PKG_ROOT / "csrc"
BUILD = PKG_ROOT / "_build"
OUT = PKG_ROOT / "pallas_flexattn" / "libflexattn.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found")
    return cand


def _flags(debug: bool) -> list[str]:
    f = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         f"-I{REPO / 'include'}", f"-I{CSRC}", "--expt-relaxed-constexpr", *ARCH]
    if debug:
        f += ["-DFA_DEBUG=1"]
    return f


def _headers() -> list[Path]:
    return list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list((REPO / "include").glob("*.h"))


def _stale(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(p.stat().st_mtime > t for p in [src, *_headers()])


def build(force: bool = False, debug: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    jobs = []
    for s in srcs:
        o = BUILD / (s.stem + ".o")
        if force or _stale(o, s):
            jobs.append((s, o))

    def run(job):
        s, o = job
        cmd = [nvcc(), *_flags(debug), "-c", str(s), "-o", str(o)]
        if verbose:
            cmd += ["-Xptxas", "-v"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {s.name}:\n{r.stderr}")
        return s.name, r.stderr

    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            for name, err in ex.map(run, jobs):
                if verbose and err:
                    print(f"--- {name}\n{err}", file=sys.stderr)
    objs = [BUILD / (s.stem + ".o") for s in srcs]
    if force or jobs or not OUT.exists():
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(OUT), *map(str, objs), "-lcudart_static", "-ldl", "-lrt",
               "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}")
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--debug", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, debug=args.debug, verbose=args.verbose))
