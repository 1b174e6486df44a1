"""Builds libomnivoice_b200.so in-tree for sm_100a.

Usage: python -m omnivoice_b200.build [--jobs N] [--verbose]

Every .cu and .cpp file under omnivoice_b200/csrc (and csrc/host) is
compiled with nvcc (`-gencode arch=compute_100a,code=sm_100a -lineinfo`)
into omnivoice_b200/_build/, then linked with the static CUDA runtime into
omnivoice_b200/libomnivoice_b200.so.  Objects are rebuilt only when a source
or any header of the library is newer than the object.
"""
from __future__ import annotations

import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
CSRC = PACKAGE / "csrc"
BUILD = PACKAGE / "_build"
LIBRARY = PACKAGE / "libomnivoice_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found; the CUDA 12.9 toolkit is required")
    return found


def sources() -> list[Path]:
    files = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))
    files += sorted((CSRC / "host").glob("*.cpp")) if (CSRC / "host").exists() else []
    return files


def headers() -> list[Path]:
    out = list((ROOT / "include").glob("*.h"))
    for pattern in ("*.hpp", "*.cuh", "*.h"):
        out += list(CSRC.rglob(pattern))
    return out


def compile_flags(source: Path) -> list[str]:
    common = ["-O3", "-std=c++20", "-Xcompiler", "-fPIC", "-I", str(ROOT / "include"),
              "-I", str(CSRC), "-I", str(CSRC / "host")]
    if source.suffix == ".cu":
        return common + ARCH + ["-lineinfo", "--expt-relaxed-constexpr",
                                "-Xptxas", "-warn-spills", "-Xcompiler", "-Wall"]
    return common + ARCH + ["-Xcompiler", "-Wall"]


def build(jobs: int = 0, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    compiler = nvcc()
    newest_header = max((h.stat().st_mtime for h in headers()), default=0.0)
    tasks = []
    objects = []
    for src in sources():
        obj = BUILD / (src.relative_to(CSRC).as_posix().replace("/", "__") + ".o")
        objects.append(obj)
        if obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, newest_header):
            continue
        tasks.append([compiler, "-c", str(src), "-o", str(obj)] + compile_flags(src))

    def run(cmd: list[str]) -> tuple[list[str], subprocess.CompletedProcess]:
        return cmd, subprocess.run(cmd, capture_output=True, text=True)

    workers = jobs or max(1, min(len(tasks), os.cpu_count() or 4))
    failed = []
    with concurrent.futures.ThreadPoolExecutor(max_workers=max(1, workers)) as pool:
        for cmd, result in pool.map(run, tasks):
            if verbose or result.returncode != 0:
                print(" ".join(cmd), file=sys.stderr)
            if result.stdout.strip() or result.stderr.strip():
                sys.stderr.write(result.stdout + result.stderr)
            if result.returncode != 0:
                failed.append(cmd[2])
    if failed:
        raise RuntimeError("compilation failed: " + ", ".join(failed))
    newest_object = max(o.stat().st_mtime for o in objects)
    if not LIBRARY.exists() or LIBRARY.stat().st_mtime < newest_object:
        link = [compiler, "-shared", "-o", str(LIBRARY)] + [str(o) for o in objects] + ARCH + [
            "-Xcompiler", "-fPIC", "-lpthread"]
        result = subprocess.run(link, capture_output=True, text=True)
        if result.returncode != 0:
            sys.stderr.write(result.stdout + result.stderr)
            raise RuntimeError("link failed")
    return LIBRARY


TESTS = ROOT / "tests" / "cpp"


def build_test_programs(verbose: bool = False) -> list[Path]:
    """Links each tests/cpp/*.cpp against the library (run by the GPU tests
    of the C++ drop-in API); binaries go to omnivoice_b200/_build/."""
    library = build(verbose=verbose)
    out = []
    for src in sorted(TESTS.glob("*.cpp")) if TESTS.exists() else []:
        exe = BUILD / src.stem
        out.append(exe)
        if exe.exists() and exe.stat().st_mtime >= max(src.stat().st_mtime, library.stat().st_mtime):
            continue
        cmd = [nvcc(), str(src), "-o", str(exe), "-O2", "-std=c++20", "-I", str(ROOT / "include"),
               "-I", str(CSRC / "host"), "-I", str(TESTS / "gufo_shim"),
               "-L", str(PACKAGE), "-lomnivoice_b200",
               "-Xlinker", "-rpath=$ORIGIN/.."] + ARCH
        result = subprocess.run(cmd, capture_output=True, text=True)
        if verbose or result.returncode != 0:
            sys.stderr.write(" ".join(cmd) + "\n" + result.stdout + result.stderr)
        if result.returncode != 0:
            raise RuntimeError(f"building {src.name} failed")
    return out


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--jobs", type=int, default=0)
    parser.add_argument("--verbose", action="store_true")
    args = parser.parse_args()
    print(build(args.jobs, args.verbose))
    for exe in build_test_programs(args.verbose):
        print(exe)


if __name__ == "__main__":
    main()
