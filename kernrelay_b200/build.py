"""Build libkernrelay.so (all CUDA kernels, the C++ runtime and the C ABI) in-tree.

The library is compiled for sm_100a only, statically links the CUDA runtime and
links NCCL dynamically (the copy that ships with torch's wheel, so a process that
already imported torch shares it).  Usage:

    python -m kernrelay_b200.build [--force] [--debug]
"""
from __future__ import annotations

import argparse
import hashlib
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
REPO = PKG.parent
INCLUDE = REPO / "include"
BUILD = PKG / "_build"
LIB = PKG / "libkernrelay.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nccl_dirs():
    import importlib.util
    spec = importlib.util.find_spec("nvidia")
    cands = []
    if spec and spec.submodule_search_locations:
        for loc in spec.submodule_search_locations:
            cands.append(Path(loc) / "nccl")
    for c in cands:
        if (c / "include" / "nccl.h").exists() and (c / "lib" / "libnccl.so.2").exists():
            return c / "include", c / "lib"
    if Path("/usr/include/nccl.h").exists():
        return Path("/usr/include"), Path("/usr/lib/x86_64-linux-gnu")
    raise RuntimeError("NCCL headers/library not found")


def _nvcc():
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found")
    return cand


def sources():
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")))


def _digest(debug: bool) -> str:
    h = hashlib.sha256()
    for p in sorted(list(CSRC.glob("*")) + list(INCLUDE.glob("*.h"))):
        if p.is_file():
            h.update(p.name.encode())
            h.update(p.read_bytes())
    h.update(b"debug" if debug else b"release")
    h.update(Path(__file__).read_bytes())
    return h.hexdigest()


def build(force: bool = False, debug: bool = False, verbose: bool = False) -> Path:
    stamp = BUILD / "stamp"
    dig = _digest(debug)
    if not force and LIB.exists() and stamp.exists() and stamp.read_text() == dig:
        return LIB
    BUILD.mkdir(parents=True, exist_ok=True)
    nvcc = _nvcc()
    nccl_inc, nccl_lib = _nccl_dirs()
    common = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler",
              "-fvisibility=hidden", f"-I{CSRC}", f"-I{INCLUDE}", f"-I{nccl_inc}",
              "--expt-relaxed-constexpr"] + ARCH
    if debug:
        common += ["-DKRB_DEBUG=1"]
    objs = []
    jobs = []
    for src in sources():
        obj = BUILD / (src.name + ".o")
        objs.append(obj)
        cmd = [nvcc] + common + ["-c", str(src), "-o", str(obj)]
        if src.suffix == ".cpp":
            # host runtime: C++20 (std::barrier for the per-device worker threads)
            cmd = [nvcc, "-x", "cu"] + common + ["-std=c++20", "-c", str(src), "-o", str(obj)]
        jobs.append(cmd)

    def run(cmd):
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("compile failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)
        if verbose:
            sys.stdout.write(r.stdout + r.stderr)

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        list(ex.map(run, jobs))
    tmp = LIB.with_suffix(".so.tmp")
    link = [nvcc, "-shared", "-o", str(tmp)] + [str(o) for o in objs] + ARCH + [
        "-cudart", "static", f"-L{nccl_lib}", "-l:libnccl.so.2",
        f"-Xlinker", f"-rpath={nccl_lib}", "-lpthread", "-ldl", "-lrt"]
    r = subprocess.run(link, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("link failed:\n" + " ".join(link) + "\n" + r.stdout + r.stderr)
    os.replace(tmp, LIB)
    stamp.write_text(dig)
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--debug", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, debug=a.debug, verbose=a.verbose))


if __name__ == "__main__":
    main()
