"""Build the sm_100a shared library ``demon_b200/libdemon_b200.so`` with nvcc.

Each ``csrc/*.cu`` is compiled to an object in parallel, then linked into one
shared library that exports the C ABI declared in ``include/demon_b200.h``.
The library is built in-tree so that it travels with the repository.

    python -m demon_b200._build            # incremental
    python -m demon_b200._build --force    # rebuild everything
    python -m demon_b200._build --ptxas-v  # print register / smem usage
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
OBJ = PKG / "_build"
LIB = PKG / "libdemon_b200.so"
SOURCES = ["capi.cu", "nvfp4_quant.cu", "nvfp4_gemm.cu", "ode_step.cu", "nvfp4_noalloc.cu", "dit_ops.cu",
           "attention.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build demon_b200")
    return cand


def _flags(ptxas_v: bool) -> list[str]:
    f = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I", str(ROOT / "include"),
                "--expt-relaxed-constexpr", "-Xcompiler", "-fvisibility=hidden"]
    if ptxas_v:
        f += ["-Xptxas", "-v"]
    return f


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list((ROOT / "include").glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def build(force: bool = False, ptxas_v: bool = False, verbose: bool = False) -> Path:
    OBJ.mkdir(exist_ok=True)
    hdr = _headers_mtime()
    jobs = []
    for s in SOURCES:
        src = CSRC / s
        obj = OBJ / (src.stem + ".o")
        if force or ptxas_v or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, hdr):
            jobs.append((src, obj))
    cc = nvcc()

    def compile_one(job):
        src, obj = job
        tmp = obj.with_suffix(f".{os.getpid()}.tmp.o")
        cmd = [cc, *_flags(ptxas_v), "-c", str(src), "-o", str(tmp)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, obj)
        return src.name, r.stderr

    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            for name, err in ex.map(compile_one, jobs):
                if (verbose or ptxas_v) and err:
                    print(f"--- {name}\n{err}", file=sys.stderr)
    objs = [OBJ / (Path(s).stem + ".o") for s in SOURCES]
    if jobs or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(f".{os.getpid()}.tmp.so")
        cmd = [cc, *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", str(tmp), *map(str, objs)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, ptxas_v=args.ptxas_v, verbose=True))


if __name__ == "__main__":
    main()
