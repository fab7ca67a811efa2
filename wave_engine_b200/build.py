"""Build the in-tree CUDA library ``wave_engine_b200/libwave_b200.so``.

Every ``csrc/*.cu`` file is compiled by nvcc for sm_100a only (B200) and
linked into one shared library exporting the C ABI of
``include/wave_b200.h``.  Objects go to ``wave_engine_b200/_build/``; a file
is recompiled when it or any header is newer than its object.

Run ``python -m wave_engine_b200.build`` or call :func:`build`.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = PKG / "_build"
LIB = PKG / "libwave_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build wave_engine_b200")


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _stale(src: Path, obj: Path, newest_header: float) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return src.stat().st_mtime > t or newest_header > t


def build(verbose: bool = False, force: bool = False, ptxas_verbose: bool = False) -> Path:
    """Compile and link the library; returns the path of the .so."""
    nvcc = _nvcc()
    BUILD.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    if not srcs:
        raise RuntimeError(f"no CUDA sources under {CSRC}")
    newest_header = max((h.stat().st_mtime for h in _headers()), default=0.0)
    jobs = []
    for s in srcs:
        o = BUILD / (s.stem + ".o")
        if force or _stale(s, o, newest_header):
            cmd = [nvcc, *ARCH, *NVCC_FLAGS, "-I", str(INCLUDE), "-I", str(CSRC), "-c", str(s), "-o", str(o)]
            if ptxas_verbose:
                cmd += ["-Xptxas", "-v"]
            jobs.append((s, cmd))

    def run(job):
        s, cmd = job
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        r = subprocess.run(cmd, capture_output=True, text=True)
        return s, r

    failed = []
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
            for s, r in ex.map(run, jobs):
                out = (r.stdout + r.stderr).strip()
                if r.returncode != 0:
                    failed.append(f"{s.name}:\n{out}")
                elif out and (verbose or ptxas_verbose):
                    print(f"[{s.name}]\n{out}", file=sys.stderr)
    if failed:
        raise RuntimeError("nvcc failed:\n" + "\n".join(failed))
    objs = [BUILD / (s.stem + ".o") for s in srcs]
    if force or jobs or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH, "-shared", "-o", str(tmp), *map(str, objs)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n" + r.stdout + r.stderr)
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, force="-f" in sys.argv, ptxas_verbose="--ptxas" in sys.argv)
    print(LIB)
