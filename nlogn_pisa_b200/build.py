"""Compile libpisa_b200.so in-tree for sm_100a with nvcc (no torch in the ABI)."""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libpisa_b200.so"
INCLUDE = ROOT / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
         "-Xcompiler", "-fvisibility=hidden"]


def sources():
    return sorted(CSRC.glob("*.cu"))


def needs_build():
    if not LIB.exists():
        return True
    stamp = LIB.stat().st_mtime
    deps = list(sources()) + list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return any(p.stat().st_mtime > stamp for p in deps)


def build(force=False, verbose=False, jobs=None, out=None, defines=()):
    """Compile every .cu into objects in parallel, then link the shared library.

    `out` and `defines` (e.g. ["PISA_LEAF_POLY_PAIRS=0"]) build a variant of
    the library elsewhere, for side-by-side measurements."""
    target = LIB if out is None else Path(out)
    if out is None and not force and not needs_build():
        return LIB
    nvcc = os.environ.get("NVCC", "nvcc")
    objdir = ROOT / "_build" if out is None else target.parent / (target.stem + "_obj")
    objdir.mkdir(parents=True, exist_ok=True)
    procs = []
    objs = []
    headers = list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    newest_header = max((p.stat().st_mtime for p in headers), default=0.0)
    for src in sources():
        obj = objdir / (src.stem + ".o")
        objs.append(obj)
        # an object is reused when it is newer than its source and every header
        if (not force and out is None and obj.exists()
                and obj.stat().st_mtime > max(src.stat().st_mtime, newest_header)):
            continue
        cmd = [nvcc, *ARCH, *FLAGS, *(f"-D{d}" for d in defines), "-I", str(INCLUDE), "-I", str(CSRC), "-c",
               str(src), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
    failed = []
    for src, p in procs:
        out, _ = p.communicate()
        text = out.decode(errors="replace")
        if p.returncode != 0:
            failed.append(f"{src.name}:\n{text}")
        elif verbose and text.strip():
            print(f"== {src.name}\n{text}")
    if failed:
        raise RuntimeError("nvcc failed:\n" + "\n".join(failed))
    tmp = target.with_suffix(".so.tmp")
    # cudart is linked statically: the library then works beside whichever
    # libcudart the host process (torch) has loaded, sharing the primary context.
    cmd = [nvcc, *ARCH, "-shared", "-cudart", "static", "-Xcompiler", "-fPIC", *map(str, objs),
           "-o", str(tmp)]
    subprocess.run(cmd, check=True)
    os.replace(tmp, target)
    return target


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
