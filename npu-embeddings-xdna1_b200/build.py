"""Build step: compile libnebw.so (CUDA, sm_100a) in-tree, and the CPU oracle.

    python npu-embeddings-xdna1_b200/build.py            # library + oracle
    python npu-embeddings-xdna1_b200/build.py --lib      # library only

The library is compiled with nvcc directly for
`-gencode arch=compute_100a,code=sm_100a`; nothing else is targeted.  The
oracle (test infrastructure) is built with oracle/Makefile: the C
restatement always, the reference's own host path only where the reference
tree exists.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
SOURCES = ["csrc/nebw.cu", "csrc/npue_file.cpp", "csrc/npue_pack.cpp"]
# every header the library includes: a change to any of them rebuilds it
DEPS = SOURCES + sorted(str(p.relative_to(PKG)) for p in (PKG / "csrc").glob("*.cuh")) + [
    "csrc/npue_file.h", "csrc/npue_pack.h", "../include/nebw.h"]
NVCC_FLAGS = ["-std=c++17", "-O3", "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo",
              "-Xcompiler", "-fPIC", "-shared"]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and Path(c).exists():
            return c
    raise FileNotFoundError("nvcc not found")


def build_lib(force: bool = False, verbose: bool = False) -> Path:
    out = PKG / "libnebw.so"
    newest = max((PKG / d).stat().st_mtime for d in DEPS)
    if out.exists() and out.stat().st_mtime >= newest and not force:
        return out
    cmd = [nvcc(), *NVCC_FLAGS, "-o", str(out), *[str(PKG / s) for s in SOURCES]]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True, cwd=PKG)
    return out


def build_host_tool(verbose: bool = False) -> Path:
    """host/nebw_embed: the C++ host side (GpuBertEncoder, the WordPiece
    tokenizer) as a file-in, file-out tool, linked against libnebw.so with an
    rpath to this dir."""
    out = PKG / "host" / "nebw_embed"
    srcs = [PKG / "host" / "nebw_embed.cpp", PKG / "host" / "gpu_bert_encoder.hpp",
            PKG / "host" / "wordpiece.cpp", PKG / "host" / "wordpiece.hpp",
            PKG / "host" / "bert_unicode.inc", REPO / "include" / "nebw.h", PKG / "libnebw.so"]
    if out.exists() and out.stat().st_mtime >= max(s.stat().st_mtime for s in srcs):
        return out
    cxx = shutil.which("g++") or "g++"
    cmd = [cxx, "-std=c++17", "-O2", "-Wall", "-I", str(REPO / "include"), "-o", str(out),
           str(PKG / "host" / "nebw_embed.cpp"), str(PKG / "host" / "wordpiece.cpp"),
           "-L", str(PKG), "-lnebw", "-Wl,-rpath,$ORIGIN/.."]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    return out


def build_oracle(verbose: bool = False):
    make = shutil.which("make")
    if not make:
        raise FileNotFoundError("make not found")
    subprocess.run([make, "-s", "-C", str(REPO / "oracle"), "port"], check=True)
    ref = Path(os.environ.get("NEBW_REFERENCE", str(REPO.parent / "reference")))
    if (ref / "runtime" / "src" / "encoders" / "bert_encoder.cpp").exists():
        subprocess.run([make, "-s", "-j8", "-C", str(REPO / "oracle"), "ref", f"REF={ref}"],
                       check=True)
        # the serving drop-in against the reference's headers and tokenizer
        # (needs libnebw.so, built first by build_lib)
        subprocess.run([make, "-s", "-C", str(REPO / "oracle"), "encoder_check", "serve_check",
                        f"REF={ref}"], check=True)


def main(argv):
    build_lib(force="--force" in argv, verbose=True)
    build_host_tool(verbose=True)
    if "--lib" not in argv:
        build_oracle(verbose=True)


if __name__ == "__main__":
    main(sys.argv[1:])
