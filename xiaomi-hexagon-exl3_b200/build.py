"""Build libexl3cu.so (sm_100a) and libexl3cu_ggml.so in-tree with nvcc.

    python xiaomi-hexagon-exl3_b200/build.py [--verbose-ptxas] [--force]

Objects go to xiaomi-hexagon-exl3_b200/_build/ (git-ignored); the two shared
libraries land next to this file so they travel with the source tree.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = PKG / "_build"
LIB = PKG / "libexl3cu.so"
GGML_LIB = PKG / "libexl3cu_ggml.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUDA_SOURCES = ["exl3cu_api.cu", "exl3cu_kernels.cu", "exl3cu_gemv.cu", "exl3cu_gemv_cluster.cu", "exl3cu_gemv_mul1.cu",
                "exl3cu_gemm_tc.cu", "exl3cu_model.cu",
                "exl3cu_hybrid.cu", "exl3cu_peers.cu"]
CXX_SOURCES = ["exl3_codec_host.cpp"]
HEADERS = ["exl3cu_internal.h", "exl3cu_decode.cuh", "exl3cu_common.cuh", "exl3cu_async.cuh", "exl3cu_mul1.cuh",
           "exl3cu_json.h"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _newer(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("build failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)
    return r.stdout + r.stderr


def build(verbose_ptxas: bool = False, force: bool = False, quiet: bool = True) -> Path:
    BUILD.mkdir(exist_ok=True)
    cc = nvcc()
    common = ["-std=c++17", "-O3", "-Xcompiler", "-fPIC,-O3", f"-I{INCLUDE}", f"-I{CSRC}"]
    hdrs = [CSRC / h for h in HEADERS] + [INCLUDE / "exl3cu.h", INCLUDE / "exl3_codec.h", INCLUDE / "exl3_model.h",
                                                 INCLUDE / "exl3cu_hybrid.h"]
    jobs = []
    for src in CUDA_SOURCES:
        obj = BUILD / (src + ".o")
        deps = [CSRC / src] + hdrs
        if force or _newer(obj, deps):
            cmd = [cc, *ARCH, "-lineinfo", *common, "-c", str(CSRC / src), "-o", str(obj)]
            if verbose_ptxas:
                cmd += ["-Xptxas", "-v"]
            jobs.append(cmd)
    for src in CXX_SOURCES:
        obj = BUILD / (src + ".o")
        if force or _newer(obj, [CSRC / src] + hdrs):
            jobs.append([cc, *common, "-x", "c++", "-c", str(CSRC / src), "-o", str(obj)])
    logs = []
    with cf.ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 1))) as ex:
        for out in ex.map(_run, jobs):
            logs.append(out)
    objs = [str(BUILD / (s + ".o")) for s in CUDA_SOURCES + CXX_SOURCES]
    if force or jobs or not LIB.exists():
        _run([cc, *ARCH, "-shared", "-o", str(LIB), *objs, "-cudart=static"])
    # ggml operator adapter (standalone build against the stand-in ggml headers)
    gsrc = CSRC / "exl3_ggml_cuda.cpp"
    if gsrc.exists() and (force or _newer(GGML_LIB, [gsrc, LIB, INCLUDE / "exl3-block.h"])):
        _run(["g++", "-std=c++17", "-O2", "-fPIC", "-shared", f"-I{INCLUDE}", f"-I{CSRC / 'ggml_stub'}",
              str(gsrc), "-o", str(GGML_LIB), f"-L{PKG}", "-lexl3cu",
              f"-Wl,-rpath,$ORIGIN"])
    if verbose_ptxas and not quiet:
        print("\n".join(logs))
    return LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose-ptxas", action="store_true")
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args(argv)
    try:
        build(verbose_ptxas=args.verbose_ptxas, force=args.force, quiet=False)
    except RuntimeError as e:
        print(e, file=sys.stderr)
        return 1
    print(f"built {LIB}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
