"""Ahead-of-time build of libmoe_b200.so for sm_100a.

    python cuda-moe-engine_b200/moe_dispatch/csrc/build.py [--force] [--verbose]

Compiles every ``*.cu`` in this directory with nvcc
(``-gencode arch=compute_100a,code=sm_100a``), in parallel, into
``<package>/lib/libmoe_b200.so``.  The CUDA runtime is linked statically so the
library does not depend on which libcudart the host process has loaded; it
shares the device's primary context (and therefore pointers and streams)
with PyTorch.  Objects go to ``_build/`` next to this file.  A source is
recompiled when it, or any header here or in ``include/``, is newer than its
object.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PACKAGE = CSRC.parent
REPO = PACKAGE.parents[1]
BUILD = CSRC / "_build"
LIBRARY = PACKAGE / "lib" / "libmoe_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr"]


def nvcc() -> str:
    for candidate in (os.environ.get("CUDA_HOME"), "/usr/local/cuda"):
        if candidate and (Path(candidate) / "bin" / "nvcc").is_file():
            return str(Path(candidate) / "bin" / "nvcc")
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found: set CUDA_HOME")
    return found


def headers():
    return list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list((REPO / "include").glob("*.h"))


def build(force: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    LIBRARY.parent.mkdir(exist_ok=True)
    compiler = nvcc()
    newest_header = max((h.stat().st_mtime for h in headers()), default=0.0)
    sources = sorted(CSRC.glob("*.cu"))
    jobs, objects = [], []
    for source in sources:
        obj = BUILD / (source.stem + ".o")
        objects.append(obj)
        stale = (
            force
            or not obj.exists()
            or obj.stat().st_mtime < max(source.stat().st_mtime, newest_header)
        )
        if stale:
            cmd = [compiler, *ARCH, *FLAGS, "-I", str(REPO / "include"), "-c", str(source), "-o", str(obj)]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
                print(" ".join(cmd), flush=True)
            jobs.append((source, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
    failed = []
    for source, job in jobs:
        out, _ = job.communicate()
        text = out.decode(errors="replace")
        if job.returncode != 0:
            failed.append(f"--- {source.name}\n{text}")
        elif verbose and text.strip():
            print(f"--- {source.name}\n{text}", flush=True)
    if failed:
        raise RuntimeError("nvcc failed:\n" + "\n".join(failed))
    if jobs or not LIBRARY.exists() or LIBRARY.stat().st_mtime < max(o.stat().st_mtime for o in objects):
        tmp = LIBRARY.with_suffix(".so.tmp")
        cmd = [compiler, *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objects)]
        result = subprocess.run(cmd, capture_output=True, text=True)
        if result.returncode != 0:
            raise RuntimeError("link failed:\n" + result.stdout + result.stderr)
        tmp.replace(LIBRARY)
    return LIBRARY


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true")
    args = parser.parse_args()
    print(build(args.force, args.verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
