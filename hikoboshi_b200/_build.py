"""Builds ``hikoboshi_b200/libhkb_mpnn.so`` in-tree for sm_100a (B200).

nvcc compiles the CUDA translation units with
``-gencode arch=compute_100a,code=sm_100a -lineinfo``; g++ compiles the plain
host C++ units.  Objects go to ``hikoboshi_b200/_build/`` and are rebuilt when
a source or header is newer.  No GPU is needed to build.
"""
from __future__ import annotations

import os
import shutil
import subprocess
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OBJ = PKG / "_build"
LIB = PKG / "libhkb_mpnn.so"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

CU_SOURCES = ["kernels_f32.cu", "kernels_tc.cu", "enc_tc.cu", "tf_tc.cu", "gemm_tc.cu", "orders.cu",
              "engine.cu", "noalloc.cu"]
CPP_SOURCES = ["host_order.cpp", "host_synth.cpp", "safetensors.cpp", "structure_io.cpp",
               "host_io.cpp"]

NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                     "-Xcompiler", "-ffp-contract=off", "--expt-relaxed-constexpr",
                     f"-I{ROOT / 'include'}", f"-I{CSRC}"]
CXX_FLAGS = ["-O2", "-std=c++17", "-fPIC", "-ffp-contract=off", "-fno-fast-math",
             "-Wall", f"-I{ROOT / 'include'}", f"-I{CSRC}", f"-I{CUDA_HOME / 'include'}"]


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.hpp")) + list(CSRC.glob("*.cuh")) + list((ROOT / "include").glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: Path, hdr_mtime: float, verbose: bool) -> Path:
    obj = OBJ / (src.name + ".o")
    if obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, hdr_mtime):
        return obj
    if src.suffix == ".cu":
        cmd = [NVCC, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    else:
        cmd = [shutil.which("g++") or "g++", *CXX_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    return obj


def build_library(verbose: bool = False) -> Path:
    OBJ.mkdir(exist_ok=True)
    hdr = _headers_mtime()
    srcs = [CSRC / s for s in CU_SOURCES + CPP_SOURCES if (CSRC / s).exists()]
    with ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, hdr, verbose), srcs))
    newest = max(o.stat().st_mtime for o in objs)
    if not LIB.exists() or LIB.stat().st_mtime < newest:
        cmd = [NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lpthread"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    build_cli(verbose)
    return LIB


CLI = PKG / "bin" / "hikoboshi"


def build_cli(verbose: bool = False) -> Path:
    """`hikoboshi design` (csrc/cli_design.cpp over include/hkb_design_api.hpp),
    linked to the in-tree library through an $ORIGIN-relative rpath."""
    src = CSRC / "cli_design.cpp"
    deps = [src, LIB, ROOT / "include" / "hkb_design_api.hpp", ROOT / "include" / "hkb_mpnn.h"]
    if CLI.exists() and CLI.stat().st_mtime >= max(d.stat().st_mtime for d in deps):
        return CLI
    CLI.parent.mkdir(exist_ok=True)
    cmd = [shutil.which("g++") or "g++", "-std=c++17", "-O2", "-Wall", f"-I{ROOT / 'include'}",
           str(src), "-o", str(CLI), f"-L{PKG}", "-lhkb_mpnn", "-Wl,-rpath,$ORIGIN/.."]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    return CLI


WEIGHTS_NAME = "Hikoboshi-ProteinMPNN-v48-020.safetensors"
WEIGHTS_SHA256 = "342b52ae248f2b70b2059313bab5ae7a358cbabac940072f71f5907eeaa21536"


def reference_root() -> Path:
    """The reference checkout: $HKB_REFERENCE_ROOT if set, else a checkout
    named ``reference`` beside this repository (it may be absent)."""
    env = os.environ.get("HKB_REFERENCE_ROOT")
    return Path(env) if env else ROOT.parent / "reference"


def stage_weights(ref_root: str | os.PathLike | None = None) -> Path:
    """Copies the reference's embedded ProteinMPNN v_48_020 weight image into
    ``hikoboshi_b200/weights/`` (SHA-256 checked) when it is not there yet."""
    import hashlib

    dst = PKG / "weights" / WEIGHTS_NAME
    if dst.exists():
        return dst
    src = Path(ref_root if ref_root is not None else reference_root()) / "weights" / WEIGHTS_NAME
    if not src.exists():
        raise FileNotFoundError(
            f"{dst} is missing and no reference checkout provides {WEIGHTS_NAME}")
    data = src.read_bytes()
    if hashlib.sha256(data).hexdigest() != WEIGHTS_SHA256:
        raise RuntimeError(f"{src}: SHA-256 mismatch")
    dst.parent.mkdir(exist_ok=True)
    dst.write_bytes(data)
    return dst


if __name__ == "__main__":
    stage_weights()
    print(build_library(verbose=True))
