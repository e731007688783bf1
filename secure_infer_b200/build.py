"""Build the native library in-tree: secure_infer_b200/_build/libsecure_infer.so.

Every CUDA source is compiled for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``); host sources go through nvcc's
host compiler.  The CUDA runtime is linked statically (nvcc's default), so the
library works next to any torch build; OpenSSL libcrypto is linked for the
host-side AES-GCM record path.

    python -m secure_infer_b200.build [--force]
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = BUILD / "libsecure_infer.so"
# Opt-in cudaMemcpyAsync interposer (LD_PRELOAD), host code only; it links
# libsecure_infer.so from its own directory and resolves the real
# cudaMemcpyAsync at run time.
INTERPOSE = BUILD / "libsecure_infer_interpose.so"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden,-O3",
          f"-I{CSRC}", f"-I{ROOT / 'include'}"]
SOURCES = ["gcm_kernels.cu", "plugin_abi.cpp", "host_runtime.cpp"]
HEADERS = ["gcm_device.cuh", "gcm_kernels.cuh", "host_runtime.h", "bitsliced_aes.cuh", "bitsliced_sbox.cuh"]


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.exists() and d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(parents=True, exist_ok=True)
    headers = [CSRC / h for h in HEADERS] + list((ROOT / "include").glob("*.h"))
    objects = []
    for src in SOURCES:
        path = CSRC / src
        if not path.exists():
            continue
        obj = BUILD / (src + ".o")
        objects.append(obj)
        if force or _stale(obj, [path, *headers]):
            cmd = [NVCC, *ARCH, *COMMON, "-c", str(path), "-o", str(obj)]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd), file=sys.stderr)
            subprocess.run(cmd, check=True)
    if force or _stale(LIB, objects):
        cmd = [NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objects), "-lcrypto", "-lpthread"]
        print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
    src = CSRC / "memcpy_interpose.cpp"
    if force or _stale(INTERPOSE, [src, LIB]):
        cxx = os.environ.get("CXX", "g++")
        cuda_inc = Path(NVCC).resolve().parent.parent / "include"
        # Export cudaMemcpyAsync alone: a preloaded library must not shadow the
        # process's C++ runtime with the copy a static libstdc++ brings along.
        script = BUILD / "interpose.map"
        script.write_text("{ global: cudaMemcpyAsync; local: *; };\n")
        cmd = [cxx, "-O2", "-std=c++17", "-fPIC", "-shared", "-fvisibility=hidden", f"-I{cuda_inc}", str(src),
               "-o", str(INTERPOSE), f"-L{BUILD}", "-lsecure_infer", "-Wl,-rpath,$ORIGIN", "-ldl",
               f"-Wl,--version-script={script}", "-Wl,--exclude-libs,ALL"]
        print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
    return LIB


def main():
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true", help="ptxas register/spill report")
    args = parser.parse_args()
    print(build(args.force, args.verbose))


if __name__ == "__main__":
    main()
