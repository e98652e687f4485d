"""Builds libstrata_cuda.so in the package directory from the .cu files here, for sm_100a only.

    python strata_mlx_b200/csrc/build.py [--jobs N] [--verbose]

Every translation unit is compiled to an object in _build/ (skipped when the object is newer than its
sources), then linked into one shared library with the CUDA runtime linked statically, so that the library
needs nothing at load time beyond the driver.
"""

import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
ROOT = os.path.dirname(PKG)
OUT = os.path.join(PKG, "libstrata_cuda.so")
BUILD = os.path.join(ROOT, "_build")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++20", "--expt-relaxed-constexpr",
         "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", "-I", os.path.join(ROOT, "include"),
         "-I", HERE]


def _deps() -> list:
    return (glob.glob(os.path.join(HERE, "*.cuh")) + glob.glob(os.path.join(HERE, "*.h"))
            + glob.glob(os.path.join(ROOT, "include", "*.h")))


# sources compiled once per block type (SC_Q2_0 .. SC_Q8_0), with the type as a macro
PER_KIND = {"matvec_kind.cu": "MV_KIND"}
KINDS = 11


def _units() -> list:
    """(source, object, extra flags) for every object of the library."""
    out = []
    for src in sorted(glob.glob(os.path.join(HERE, "*.cu"))):
        name = os.path.basename(src)
        if name in PER_KIND:
            for k in range(KINDS):
                out.append((src, os.path.join(BUILD, f"{name}.{k}.o"), [f"-D{PER_KIND[name]}={k}"]))
        else:
            out.append((src, os.path.join(BUILD, name + ".o"), []))
    return out


def _compile(unit: tuple, verbose: bool, extra: list) -> str:
    src, obj, defs = unit
    newest = max(os.path.getmtime(p) for p in [src, *_deps()])
    if os.path.exists(obj) and os.path.getmtime(obj) >= newest and not extra:
        return obj
    cmd = [NVCC, *FLAGS, *defs, *extra, "-c", src, "-o", obj]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
    if verbose and r.stderr:
        print(r.stderr, flush=True)
    return obj


def build(jobs: int = 8, verbose: bool = False, extra: list | None = None) -> str:
    os.makedirs(BUILD, exist_ok=True)
    import importlib.util

    spec = importlib.util.spec_from_file_location("sc_gen_tables", os.path.join(HERE, "gen_tables.py"))
    gen_tables = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(gen_tables)

    gen_tables.main(os.path.join(HERE, "iq_tables.h"))
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(lambda u: _compile(u, verbose, extra or []), _units()))
    newest = max(os.path.getmtime(o) for o in objs)
    if not os.path.exists(OUT) or os.path.getmtime(OUT) < newest or extra:
        cmd = [NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-cudart", "static", *objs, "-o", OUT,
               "-lcuda"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--jobs", type=int, default=os.cpu_count() or 4)
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers / spills / shared memory per kernel")
    a = ap.parse_args()
    print(build(a.jobs, a.verbose, ["-Xptxas", "-v"] if a.ptxas_info else None))
