"""Build the CPU oracle ``oracle/libwave_oracle.so`` from ``wave_oracle.c``
(the attention path) and ``serve_oracle.c`` (the serve-tier layer around it).

The oracle is test infrastructure (the parity checker and the timed CPU
baseline).  It is compiled with -ffp-contract=off so that, like rustc, the
compiler never fuses a multiply and an add, and it links glibc libm for
atan2f/cosf/expf/logf/fmodf exactly as Rust's f32 methods do on Linux.

The reference implementation itself (Rust crate wave-engine) cannot be built
here: no Rust toolchain, and its path dependency ../kerr-memory is absent.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "wave_oracle.c"
SRCS = [SRC, HERE / "serve_oracle.c"]
LIB = HERE / "libwave_oracle.so"
CFLAGS = ["-O2", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared", "-pthread", "-std=c11"]


def build(force: bool = False) -> Path:
    if not force and LIB.exists() and all(LIB.stat().st_mtime >= src.stat().st_mtime for src in SRCS):
        return LIB
    cc = os.environ.get("CC", "gcc")
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [cc, *CFLAGS, *[str(src) for src in SRCS], "-o", str(tmp), "-lm"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + r.stdout + r.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="-f" in sys.argv))
