"""Build libltxattn_cuda.so in-tree with nvcc for sm_100a.

    python ltx-2.5-swift_b200/build.py          # incremental
    python ltx-2.5-swift_b200/build.py --force  # rebuild everything

Objects go to ``_build/`` beside this file; the shared library lands next to
this file, where ``ltxattn`` loads it.  The CUDA runtime is linked statically
so the library does not depend on which libcudart a host process loaded;
NCCL is opened at run time (``csrc/comm.cpp``).
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import re
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
LIB = os.path.join(HERE, "libltxattn_cuda.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
                     "-Xcompiler", "-fvisibility=hidden", "-I", CSRC, "-I", INCLUDE]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return cand


def _headers():
    return glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


# Kernels that re-split registers between warpgroups (setmaxnreg) must be
# launched with exactly the per-thread count their split was sized for: a
# setmaxnreg.inc that asks for more than the launch provided never returns.
# ptxas' report is checked against the value the kernel source assumes.
REGISTER_PINS = {"fwd_sm100.cu": ("fwd_bf16_sm100_kernel", 168),
                 "fwd_short_sm100.cu": ("fwd_short_sm100_kernel", 128),
                 "fwd_persist_sm100.cu": ("fwd_persist_sm100_kernel", 168)}


def _check_register_pin(src: str, ptxas_log: str) -> None:
    pin = REGISTER_PINS.get(os.path.basename(src))
    if not pin:
        return
    kernel, regs = pin
    lines = ptxas_log.splitlines()
    found = 0
    for i, ln in enumerate(lines):
        if "Compiling entry function" in ln and kernel in ln:
            for ln2 in lines[i + 1:i + 6]:
                m = re.search(r"Used (\d+) registers", ln2)
                if m:
                    found += 1
                    if int(m.group(1)) != regs:
                        raise RuntimeError(f"{kernel}: ptxas used {m.group(1)} registers, the warpgroup "
                                           f"register split assumes {regs}")
                    break
    if not found:
        raise RuntimeError(f"{kernel}: no ptxas register report found")


def _compile(src: str, obj: str, verbose: bool) -> str:
    cmd = [nvcc()] + NVCC_FLAGS + ["-Xptxas=-v", "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")
    _check_register_pin(src, r.stderr + r.stdout)
    return r.stderr if verbose else ""


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    headers = _headers()
    jobs = []
    objs = []
    for src in sources:
        obj = os.path.join(OBJ, os.path.basename(src) + ".o")
        objs.append(obj)
        if force or _stale(obj, [src] + headers):
            jobs.append((src, obj))
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(8, len(jobs))) as ex:
            for msg in ex.map(lambda j: _compile(j[0], j[1], verbose), jobs):
                if verbose and msg:
                    print(msg, file=sys.stderr)
    if force or jobs or _stale(LIB, objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-o", LIB] + objs + ["-cudart", "static", "-ldl", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
