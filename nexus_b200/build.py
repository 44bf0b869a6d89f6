"""Build the sm_100a backend library ``nexus_b200/libnexus_cuda.so`` in-tree.

Every CUDA translation unit is compiled with
``-gencode arch=compute_100a,code=sm_100a -lineinfo``; the bit-exact block
format kernels (kernels_quant.cu) additionally with ``-fmad=false`` and the
host code with ``-ffp-contract=off`` so their arithmetic rounds like the
reference.  nvcc cross-compiles without a GPU.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
BUILD = HERE / "_build"
LIB = HERE / "libnexus_cuda.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

CU_COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-ffp-contract=off",
             "--expt-relaxed-constexpr", "-Xptxas", "-v"] + ARCH
UNITS = {
    "kernels_quant.cu": ["-fmad=false"],
    "kernels_gemv.cu": [],
    "kernels_gemv_q4k.cu": [],
    "kernels_gemv_q80.cu": [],
    "kernels_gemv_q40.cu": [],
    "kernels_gemv_q2k.cu": [],
    "kernels_gemm.cu": [],
    "kernels_attn.cu": [],
    "kernels_attn_pk.cu": [],
    "kernels_attn_prefill.cu": [],
    "kernels_step.cu": [],
    "kernels_peer.cu": [],
    "kernels_misc.cu": [],
    "engine.cu": [],
    "noalloc.cu": [],
}
CXX_UNITS = ["host.cpp", "scheduler.cpp"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _run(cmd: list[str], log: Path) -> None:
    res = subprocess.run(cmd, capture_output=True, text=True)
    log.write_text(res.stdout + res.stderr)
    if res.returncode != 0:
        raise RuntimeError(f"build failed: {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")


def sources() -> list[Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")) + list(CSRC.glob("*.cuh"))
                  + list(CSRC.glob("*.h")) + [HERE.parent / "include" / "nexus_cuda.h"])


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in sources() + [Path(__file__)])


def build(force: bool = False, verbose: bool = False, out: Path | None = None, build_dir: Path | None = None,
          extra_cu_flags: list[str] | None = None) -> Path:
    """Compile the library (into `out`, default nexus_b200/libnexus_cuda.so);
    extra_cu_flags are added to every CUDA unit (e.g. -DNX_GEMV_WARPS=16)."""
    lib_out = Path(out) if out else LIB
    bdir = Path(build_dir) if build_dir else BUILD
    if out is None and not force and not extra_cu_flags and up_to_date():
        return LIB
    bdir.mkdir(parents=True, exist_ok=True)
    nv = nvcc()
    jobs = []
    objs = []
    for unit, extra in UNITS.items():
        obj = bdir / (unit + ".o")
        objs.append(obj)
        jobs.append(([nv, "-c", str(CSRC / unit), "-o", str(obj)] + CU_COMMON + extra + list(extra_cu_flags or []),
                     bdir / (unit + ".log")))
    for unit in CXX_UNITS:
        obj = bdir / (unit + ".o")
        objs.append(obj)
        jobs.append((["g++", "-c", str(CSRC / unit), "-o", str(obj), "-O2", "-std=c++17", "-fPIC",
                      "-ffp-contract=off", "-fno-fast-math", "-I/usr/local/cuda/include"], bdir / (unit + ".log")))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        futs = [ex.submit(_run, cmd, log) for cmd, log in jobs]
        for f in futs:
            f.result()
    tmp = lib_out.with_suffix(".so.tmp")
    _run([nv, "-shared", "-o", str(tmp)] + [str(o) for o in objs] + ARCH + ["-lpthread"], bdir / "link.log")
    os.replace(tmp, lib_out)
    if verbose:
        for unit in UNITS:
            print((bdir / (unit + ".log")).read_text())
    return lib_out


if __name__ == "__main__":
    import argparse

    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", action="store_true")
    ap.add_argument("--out", default=None, help="output library path")
    ap.add_argument("--build-dir", default=None)
    ap.add_argument("-D", action="append", default=[], help="extra CUDA define, e.g. -D NX_GEMV_WARPS=16")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.v, out=a.out, build_dir=a.build_dir, extra_cu_flags=[f"-D{d}" for d in a.D]))
