"""Build libzenith_ssd.so in-tree with nvcc for sm_100a (no torch headers involved).

    python -m zenith_b200.build          # or __graft_entry__.build()
"""
from __future__ import annotations

import os
import pathlib
import subprocess
import sys

PKG = pathlib.Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libzenith_ssd.so"
SOURCES = ["capi.cu", "capi_noalloc.cu", "ssd_simt.cu", "ssd_tc.cu", "mamba3_layer.cu", "ssd_decode.cu", "lm_kernels.cu", "wait_probe.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or "/usr/local/cuda/bin/nvcc"
    return cand if os.path.exists(cand) else "nvcc"


def needs_build() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = list(CSRC.glob("*")) + list((ROOT / "include").glob("*.h"))
    return any(p.stat().st_mtime > t for p in deps)


def build(verbose: bool = False, force: bool = False) -> pathlib.Path:
    if not force and not needs_build():
        return LIB
    objs = []
    build_dir = PKG / "_build"
    build_dir.mkdir(exist_ok=True)
    procs = []
    for src in SOURCES:
        obj = build_dir / (src + ".o")
        cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
               "-I", str(ROOT / "include"), "-I", str(CSRC), "--expt-relaxed-constexpr", "-c", str(CSRC / src), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        procs.append((cmd, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
        objs.append(obj)
    failed = False
    for cmd, pr in procs:
        out, _ = pr.communicate()
        if out and (verbose or pr.returncode):
            sys.stderr.write(out)
        if pr.returncode:
            failed = True
            sys.stderr.write("FAILED: " + " ".join(cmd) + "\n")
    if failed:
        raise RuntimeError("nvcc failed")
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", str(tmp), *map(str, objs), "-lcudart_static", "-lrt", "-ldl", "-lpthread"]
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, force=True)
    print(LIB)
