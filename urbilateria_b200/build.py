"""Build liburb_moe (the C-ABI library) in-tree for sm_100a.

    python -m urbilateria_b200.build        # or __graft_entry__.build()

Steps: (1) generate the libm exception tables once (gen_expf_table.c, ~90 s on 8 cores;
gen_log1pf_table.c, ~10 s),
(2) compile every csrc/*.cu with nvcc for sm_100a, (3) link urbilateria_b200/liburb_moe.so
(static CUDA runtime) and urbilateria_b200/liburb_moe.a (for a Rust build.rs).
Objects are cached under urbilateria_b200/_build keyed by source modification time.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
GEN = os.path.join(CSRC, "_gen")
TABLE = os.path.join(GEN, "expf_table.bin")
LOG1P_TABLE = os.path.join(GEN, "log1pf_table.bin")
SO = os.path.join(PKG, "liburb_moe.so")
AR = os.path.join(PKG, "liburb_moe.a")

CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
                     "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr",
                     "-I", os.path.join(ROOT, "include")]
HOST_CXX = "/usr/bin/g++"
HOST_CC = "/usr/bin/gcc"


def _run(cmd, **kw):
    r = subprocess.run(cmd, capture_output=True, text=True, **kw)
    if r.returncode != 0:
        raise RuntimeError("command failed: %s\n%s\n%s" % (" ".join(cmd), r.stdout, r.stderr))
    return r


def _stale(out, deps):
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def _libm_table(out: str, gen_src: str) -> str:
    os.makedirs(GEN, exist_ok=True)
    src = os.path.join(CSRC, gen_src)
    if not _stale(out, [src]):
        return out
    exe = os.path.join(GEN, os.path.splitext(gen_src)[0])
    _run([HOST_CC, "-O2", "-fopenmp", src, "-o", exe, "-lm"])
    tmp = out + ".tmp"
    _run([exe, tmp])
    os.replace(tmp, out)
    return out


def expf_table() -> str:
    return _libm_table(TABLE, "gen_expf_table.c")


def log1pf_table() -> str:
    return _libm_table(LOG1P_TABLE, "gen_log1pf_table.c")


def build(verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    table = expf_table()
    log1p_table = log1pf_table()
    headers = glob.glob(os.path.join(CSRC, "*.cuh")) + [os.path.join(ROOT, "include", "urb_moe.h")]
    jobs = []
    for cu in sorted(glob.glob(os.path.join(CSRC, "*.cu"))):
        obj = os.path.join(BUILD, os.path.basename(cu) + ".o")
        jobs.append((obj, [NVCC] + NVCC_FLAGS + ["-c", cu, "-o", obj], [cu] + headers))
    cpp = os.path.join(CSRC, "expf_table.cpp")
    obj = os.path.join(BUILD, "expf_table.cpp.o")
    jobs.append((obj, [HOST_CXX, "-O2", "-std=c++17", "-fPIC", "-fvisibility=hidden",
                       "-I", os.path.join(CUDA_HOME, "include"), "-I", os.path.join(ROOT, "include"),
                       '-DURB_EXPF_TABLE_PATH=%s' % table,
                       '-DURB_LOG1PF_TABLE_PATH=%s' % log1p_table, "-c", cpp, "-o", obj],
                 [cpp, table, log1p_table] + headers))
    todo = [j for j in jobs if _stale(j[0], j[2])]
    with cf.ThreadPoolExecutor(max_workers=max(1, os.cpu_count() or 1)) as ex:
        for f in [ex.submit(_run, cmd) for _, cmd, _ in todo]:
            r = f.result()
            if verbose and r.stderr:
                print(r.stderr, file=sys.stderr)
    objs = [j[0] for j in jobs]
    if _stale(SO, objs):
        tmp = SO + ".tmp"
        _run([NVCC] + ARCH + ["-shared", "-o", tmp] + objs + ["-lcudart_static", "-lrt", "-lpthread", "-ldl"])
        os.replace(tmp, SO)
    if _stale(AR, objs):
        if os.path.exists(AR):
            os.remove(AR)
        _run(["ar", "rcs", AR] + objs)
    return SO


def clean():
    shutil.rmtree(BUILD, ignore_errors=True)
    for p in (SO, AR):
        if os.path.exists(p):
            os.remove(p)


if __name__ == "__main__":
    print(build(verbose=True))
