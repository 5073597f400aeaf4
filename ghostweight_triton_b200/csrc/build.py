"""Build recipe for libghostweight_b200.so (sm_100a only).

Compiles every ``*.cu`` in this directory with nvcc for ``sm_100a`` and links
them into ``ghostweight_triton_b200/libghostweight_b200.so`` (in-tree, so the
built library travels with the source tree). No torch headers are involved:
the library exports a plain C ABI (include/ghostweight_b200.h).

Usage: ``python -m ghostweight_triton_b200.csrc.build [--force] [--verbose]``
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PKG = CSRC.parent
REPO = PKG.parent
INCLUDE = REPO / "include"
BUILD_DIR = REPO / "_build" / "csrc"
LIB_NAME = "libghostweight_b200.so"
LIB_PATH = PKG / LIB_NAME

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden",
    "-Xptxas", "-warn-spills",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC or install the CUDA toolkit)")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False, extra_flags: list[str] | None = None) -> Path:
    """Compile (if stale) and return the path of the shared library."""
    nvcc = _nvcc()
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    headers = _headers()
    objs: list[Path] = []
    jobs = []
    flags = NVCC_FLAGS + list(extra_flags or [])
    for src in sources():
        obj = BUILD_DIR / (src.stem + ".o")
        objs.append(obj)
        if force or _stale(obj, [src, *headers, Path(__file__)]):
            cmd = [nvcc, *ARCH_FLAGS, *flags, f"-I{INCLUDE}", "-c", str(src), "-o", str(obj)]
            jobs.append(cmd)

    def run(cmd: list[str]) -> tuple[list[str], subprocess.CompletedProcess]:
        return cmd, subprocess.run(cmd, capture_output=True, text=True)

    if jobs:
        workers = max(1, min(len(jobs), os.cpu_count() or 1))
        with cf.ThreadPoolExecutor(max_workers=workers) as ex:
            for cmd, res in ex.map(run, jobs):
                if verbose or res.returncode != 0:
                    sys.stderr.write(" ".join(cmd) + "\n" + res.stdout + res.stderr)
                if res.returncode != 0:
                    raise RuntimeError(f"nvcc failed on {cmd[-3]}")
    if force or jobs or _stale(LIB_PATH, objs):
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-Xlinker", f"-soname={LIB_NAME}", "-o", str(LIB_PATH),
               *map(str, objs)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if verbose or res.returncode != 0:
            sys.stderr.write(" ".join(cmd) + "\n" + res.stdout + res.stderr)
        if res.returncode != 0:
            raise RuntimeError("link of libghostweight_b200.so failed")
    build_fast(force=force, verbose=verbose)
    return LIB_PATH


FAST_SRC = CSRC / "gw_pyfast.c"


def fast_module_path() -> Path:
    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    return PKG / f"_gwfast{suffix}"


def build_fast(force: bool = False, verbose: bool = False) -> Path | None:
    """Compile the CPython fast-call bindings (gw_pyfast.c) against libghostweight_b200.so.

    Plain C against the Python headers (no torch), linked to the library in this
    directory through an $ORIGIN run path. Returns None (the ctypes binding is
    used instead) when no C compiler or no Python headers are available.
    """
    out = fast_module_path()
    cc = os.environ.get("CC") or shutil.which("gcc") or shutil.which("cc")
    inc = sysconfig.get_paths().get("include")
    if not cc or not inc or not (Path(inc) / "Python.h").exists():
        return None
    if not force and not _stale(out, [FAST_SRC, LIB_PATH, INCLUDE / "ghostweight_b200.h", Path(__file__)]):
        return out
    cmd = [cc, "-O2", "-shared", "-fPIC", "-std=c11", f"-I{inc}", f"-I{INCLUDE}", str(FAST_SRC),
           f"-L{PKG}", "-l:" + LIB_NAME, "-Wl,-rpath,$ORIGIN", "-o", str(out)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or res.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + res.stdout + res.stderr)
    if res.returncode != 0:
        raise RuntimeError("build of the fast-call bindings failed")
    return out


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true", help="pass -Xptxas -v")
    args = ap.parse_args()
    extra = ["-Xptxas", "-v"] if args.ptxas_verbose else []
    print(build(force=args.force or args.ptxas_verbose, verbose=args.verbose or args.ptxas_verbose,
                extra_flags=extra))


if __name__ == "__main__":
    main()
