"""Build libsinkattn.so in-tree with nvcc for sm_100a (B200).

Usage: python -m sinkattn_b200.build [--verbose] [--force]

Each csrc/*.cu file is compiled to an object under sinkattn_b200/_build/ and
linked into sinkattn_b200/libsinkattn.so. The build is incremental on file
modification times (sources and headers) and needs no GPU.
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
INCLUDE = PKG.parent / "include"
BUILD = PKG / "_build"
LIB = PKG / "libsinkattn.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-I",
    str(INCLUDE),
]


def find_nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError(f"nvcc not found (looked for {cand})")
    return cand


def _newest_dep_mtime() -> float:
    deps = list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return max((p.stat().st_mtime for p in deps), default=0.0)


def _compile(nvcc: str, src: Path, obj: Path, extra: list[str], verbose: bool) -> None:
    cmd = [nvcc, *ARCH_FLAGS, *COMMON_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr, flush=True)


def build(verbose: bool = False, force: bool = False) -> Path:
    """Compile every CUDA source and link the shared library; returns its path."""
    nvcc = find_nvcc()
    BUILD.mkdir(exist_ok=True)
    extra: list[str] = []
    if verbose:
        extra += ["-Xptxas", "-v"]
    stamp = BUILD / "flags.txt"
    flag_str = " ".join(ARCH_FLAGS + COMMON_FLAGS + extra)
    if not stamp.exists() or stamp.read_text() != flag_str:
        force = True
        stamp.write_text(flag_str)
    dep_time = _newest_dep_mtime()
    jobs = []
    objs = []
    for src in sorted(CSRC.glob("*.cu")):
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        if force or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, dep_time):
            jobs.append((src, obj))
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            futs = [ex.submit(_compile, nvcc, s, o, extra, verbose) for s, o in jobs]
            for f in futs:
                f.result()
    if jobs or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args(argv)
    path = build(verbose=args.verbose, force=args.force)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
