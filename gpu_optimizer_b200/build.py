"""Build libgpo.so (the sm_100a kernel library) in-tree with nvcc.

Usage: ``python -m gpu_optimizer_b200.build [--jobs N] [--verbose]``.

Every ``csrc/*.cu`` translation unit is compiled for ``sm_100a`` in parallel
into ``_build/`` at the repository root, the kernel sources are embedded for
``gpo_source`` (``_build/gpo_sources.inc``), and the objects are linked with
the static CUDA runtime into ``gpu_optimizer_b200/libgpo.so``.  A unit is
rebuilt only when it, or a header it includes, is newer than its object.
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
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = ROOT / "_build"
LIB = PKG / "libgpo.so"
HEADERS = [CSRC / "gpo_common.cuh", CSRC / "gpo_internal.h", ROOT / "include" / "gpo.h"]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    *ARCH, "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr",
    "-DNDEBUG", f"-I{BUILD}", f"-I{ROOT / 'include'}",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; the sm_100a kernel library cannot be built")


def _sources_inc() -> Path:
    """Write the embedded-source table used by gpo_source()."""
    BUILD.mkdir(exist_ok=True)
    out = BUILD / "gpo_sources.inc"
    parts = ["struct SourceEntry { const char* name; const char* text; };\n",
             "static const SourceEntry kSources[] = {\n"]
    for f in sorted([*CSRC.glob("*.cu"), *CSRC.glob("*.cuh")]):
        if f.stem == "abi":
            continue
        text = f.read_text()
        chunks = [text[i:i + 4000] for i in range(0, len(text), 4000)] or [""]
        lits = "\n".join(f'R"gposrc({c})gposrc"' for c in chunks)
        parts.append(f'  {{"{f.stem}", {lits}}},\n')
    parts.append("};\n")
    new = "".join(parts)
    if not out.exists() or out.read_text() != new:
        out.write_text(new)
    return out


def _stale(obj: Path, src: Path, deps: list[Path]) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(p.stat().st_mtime > t for p in [src, *deps] if p.exists())


def build(jobs: int | None = None, verbose: bool = False, force: bool = False) -> Path:
    """Compile and link libgpo.so; returns its path."""
    exe = nvcc()
    inc = _sources_inc()
    srcs = sorted(CSRC.glob("*.cu"))
    objs = []
    todo = []
    for s in srcs:
        o = BUILD / (s.stem + ".o")
        objs.append(o)
        deps = HEADERS + ([inc] if s.stem == "abi" else [])
        if force or _stale(o, s, deps):
            todo.append((s, o))

    def compile_one(item):
        s, o = item
        cmd = [exe, *NVCC_FLAGS, "-c", str(s), "-o", str(o)]
        if verbose:
            cmd += ["-Xptxas", "-v"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        return s, r

    failed = []
    with ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as ex:
        for s, r in ex.map(compile_one, todo):
            if verbose and (r.stdout or r.stderr):
                print(r.stdout + r.stderr, file=sys.stderr)
            if r.returncode != 0:
                failed.append((s, r.stdout + r.stderr))
    if failed:
        msg = "\n".join(f"--- {s.name}\n{log}" for s, log in failed)
        raise RuntimeError(f"nvcc failed:\n{msg}")
    if todo or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [exe, *ARCH, "-shared", "-cudart", "static", "-o", str(tmp),
               *map(str, objs), "-lpthread", "-ldl", "-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(a.jobs, a.verbose, a.force))


if __name__ == "__main__":
    main()
